"""QwenBackbone on B200: the reference's forward with every per-layer row op
on libqdc_b200's sm_100a kernels, and every intermediate in the model's
libqdc_b200 workspace arena.

Public API, mirroring src/backbone.jl:
  QwenBackbone.from_directory(dir, device)   QwenBackbone(dir; device), :74-192
  backbone_hidden(b, ids, mask[, positions])  :433-460 (host float32 (tokens, hidden))
  backbone_last_hidden(b, ids, mask)          :470-490
  batch_backbone_hidden(b, ids, mask)         the batched hook of :66-70: each
                                              row's last-position state, host
                                              (batch, hidden)
  batch_hidden(b, ids, mask)                  many equal-length sequences in one
                                              pass; device (B*S, hidden)

Per layer (native_layer, src/backbone.jl:363-382):
  input norm   -- qdc gather+norm for layer 0, else fused into the previous
                  layer's MLP residual add (qdc_residual_rms)
  attention    -- full: one [q;k;v] GEMM, qdc q/k norm + partial RoPE,
                  causal GQA attention (batched GEMMs and a softmax over
                  materialised scores, as ext/cuda_attention.jl:163-175), qdc
                  sigmoid gate read from the attention output in place, o GEMM;
                  delta: one [qkv;z;a;b] GEMM, qdc causal 4-tap conv + SiLU +
                  q/k L2 norms, qdc beta/decay gates, chunked gated delta
                  rule (torch GEMMs + the qdc unit-lower-triangular solve),
                  qdc gated norm reading z in place, out GEMM
  post norm    -- qdc residual add + RMSNorm
  MLP          -- one [gate;up] GEMM, qdc SwiGLU, down GEMM
  residual add -- fused with the next layer's input norm / the final norm.

Memory (ext/cuda_workspace.jl:4-87): each model owns a libqdc_b200 context
whose arena holds every intermediate of a forward (workspace.py).  The
arena is sized once per shape (forward_bytes), the cursor is reset at the
start of each forward, and each layer releases its slots when it ends, so
layers of one kind carve the same slots forward after forward and a
captured graph replays the addresses it was recorded against.  Every torch
op of the forward writes into those slots (out=, in-place ops), so after
warm-up a forward allocates no device memory.

The projections, attention, conv and delta rule are the reference's
out-of-scope parts; they run as plain torch Float32 ops (cuBLAS GEMMs with
TF32 disabled, as the reference computes in Float32, src/backbone.jl:14-16).
"""

import collections
import math
import os

import numpy as np
import torch

from . import ops
from ._lib import ArgumentError
from .model import Config, device_f32, load_weights, pack_layers, random_weights
from .workspace import Workspace, slot_bytes, spec_bytes

FLOATMAX32 = float(np.finfo(np.float32).max)
MAX_GRAPHS = 32  # cached last-token graphs per model (shapes beyond evict the oldest)
MAX_CONSTS = 8  # cached causal masks per model (one per sequence length in use)
DELTA_CHUNK = 64  # src/backbone.jl:301, ext/cuda_delta_chunked.jl:9
SCAN_MAX_HEADS = 64  # batch x value heads up to which the delta hand-off runs as a linear scan
ATTN_SCORE_BYTES = 1 << 30  # attention scores per chunk of sequences (one buffer)
F32 = torch.float32


def _device_f32(x, device):
    return device_f32(x, device)


def check_sequence(vocab, ids, mask):
    """src/backbone.jl:413-422."""
    if len(ids) != len(mask):
        raise ArgumentError(1, "Input IDs and mask must have identical lengths.")
    if len(ids) == 0:
        raise ArgumentError(1, "Inputs must not be empty.")
    ids_a = np.asarray(ids)
    if ids_a.min() < 0 or ids_a.max() >= vocab:
        raise ArgumentError(2, "Token ID is outside the vocabulary.")
    m = np.asarray(mask)
    if not np.isin(m, (0, 1)).all():
        raise ArgumentError(1, "Mask values must be zero or one.")


# ----------------------------------------------------------- slot specs
# The slots each part of the forward carves, in carve order: name ->
# (shape, dtype).  The forward takes exactly these (Workspace.take_all) and
# forward_bytes sums them, so the arena is sized by the same description.

def _spec(**slots):
    return {k: (v, F32) if isinstance(v[0], int) else v for k, v in slots.items()}


def _root_spec(cfg, B, S, full_mask, host_mask, has_full):
    T, H = B * S, cfg.hidden
    spec = _spec(x=(T, H), r=(T, H), y=(T, H))
    if host_mask:
        spec["mask"] = ((T,), torch.int32)
    if not full_mask:
        spec["maskf"] = ((T,), F32)
        if has_full:
            spec["key_off"] = ((B, S), torch.bool)
            spec["notallowed"] = ((B, S, S), torch.bool)
    return spec


def _attn_chunk(cfg, B, Sq, S):
    """Sequences per attention chunk: their scores fit ATTN_SCORE_BYTES."""
    return max(1, min(B, ATTN_SCORE_BYTES // max(cfg.heads * Sq * S * 4, 1)))


def _attend_spec(cfg, nb, Sq, S):
    D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    G = Hq // Hkv
    return _spec(qh=(nb, Hq, Sq, D), kh=(nb, Hkv, S, D), vh=(nb, Hkv, S, D),
                 scores=(nb * Hkv, G * Sq, S), probs=(nb * Hkv, G * Sq, S), values=(nb, Hq, Sq, D))


def _full_spec(cfg, B, S):
    T, D, Hq, Hkv = B * S, cfg.head_dim, cfg.heads, cfg.kv_heads
    spec = _spec(proj=(T, Hq * 2 * D + 2 * Hkv * D), q=(T, Hq, D), k=(T, Hkv, D))
    spec.update(_attend_spec(cfg, _attn_chunk(cfg, B, S, S), S, S))
    spec.update(_spec(gated=(T, Hq * D), out=(T, cfg.hidden)))
    return spec


def _full_last_spec(cfg, B, S):
    T, D, Hq, Hkv = B * S, cfg.head_dim, cfg.heads, cfg.kv_heads
    spec = _spec(kv=(T, 2 * Hkv * D), qgate=(B, Hq * 2 * D), q=(B, Hq, D), k=(T, Hkv, D))
    spec.update(_attend_spec(cfg, B, 1, S))
    spec.update(_spec(gated=(B, Hq * D), out=(B, cfg.hidden)))
    return spec


def _chunked_spec(B, S, Hv, Dk, Dv, scan, C=DELTA_CHUNK):
    n = -(-S // C)
    S2, BH = n * C, B * Hv
    spec = _spec(Qh=(B, Hv, S2, Dk), Kh=(B, Hv, S2, Dk), Vh=(B, Hv, S2, Dv), bet=(B, Hv, S2),
                 cum=(B, Hv, S2), e=(B, Hv, S2), be=(B, Hv, S2), tail=(B, Hv, S2),
                 pair=(B, Hv, n, C, C), system=(B, Hv, n, C, C), intra=(B, Hv, n, C, C),
                 X=(B, Hv, n, C, Dv + Dk), qe=(B, Hv, n, C, Dk), ending=(B, Hv, n, C, Dk),
                 final=(B, Hv, n), U=(B, Hv, n, C, Dv))
    if scan:
        spec.update(_spec(A=(B, Hv, n, Dk, Dk), Bc=(B, Hv, n, Dv, Dk), states=(B, Hv, n, Dv, Dk)))
    else:
        spec.update(_spec(state=(BH, Dv, Dk), corr=(BH, C, Dv)))
    return spec


def _delta_spec(cfg, B, S, full_mask):
    T, H = B * S, cfg.hidden
    Hk, Hv, Dk, Dv = cfg.key_heads, cfg.value_heads, cfg.key_dim, cfg.value_dim
    spec = {} if full_mask else _spec(masked=(T, H))
    spec.update(_spec(proj=(T, cfg.qkv_width + cfg.value_width + 2 * Hv), q=(T, Hk, Dk), k=(T, Hk, Dk),
                      v=(T, Hv, Dv), beta=(T, Hv), decay=(T, Hv)))
    spec.update(_chunked_spec(B, S, Hv, Dk, Dv, B * Hv <= SCAN_MAX_HEADS))
    spec.update(_spec(o=(B, S, Hv, Dv), gated=(T, Hv * Dv), out=(T, H)))
    return spec


def _mlp_spec(cfg, rows):
    I = cfg.intermediate
    return _spec(gate_up=(rows, 2 * I), h=(rows, I), mlp=(rows, cfg.hidden))


def forward_bytes(cfg, B, S, full_mask, host_mask, last_only):
    """Arena bytes of one forward: the root slots plus the largest layer
    (each layer releases its slots when it ends)."""
    kinds = set(cfg.layer_types)
    has_full = "full_attention" in kinds
    root = spec_bytes(_root_spec(cfg, B, S, full_mask, host_mask, has_full))
    T = B * S
    peak = 0
    if has_full:
        peak = max(peak, spec_bytes(_full_spec(cfg, B, S)) + spec_bytes(_mlp_spec(cfg, T)))
    if "linear_attention" in kinds:
        peak = max(peak, spec_bytes(_delta_spec(cfg, B, S, full_mask)) + spec_bytes(_mlp_spec(cfg, T)))
    if last_only:
        last = cfg.layer_types[-1]
        attn = _full_last_spec(cfg, B, S) if last == "full_attention" else _delta_spec(cfg, B, S, full_mask)
        peak = max(peak, spec_bytes(attn) + 2 * slot_bytes((B, cfg.hidden)) + spec_bytes(_mlp_spec(cfg, B)))
    return root + peak


# ------------------------------------------------------------- the model

class QwenBackbone:
    def __init__(self, config, weights, device="cuda"):
        self.config = config
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ArgumentError(1, "QwenBackbone(…; device) needs a CUDA device: the per-layer "
                                   "kernels have no CPU path")
        # the model's own context: its workspace arena holds every
        # intermediate of a forward (ext/cuda_workspace.jl:4-46)
        self.ctx = ops.Context(self.device)
        self.ws = Workspace(self.ctx)
        self.embedding = _device_f32(weights["embed_tokens.weight"], self.device)
        self.final_norm = _device_f32(weights["norm.weight"], self.device)
        self.layers = pack_layers(config, weights, self.device)
        self._init_caches()

    def _init_caches(self):
        self._rope = {}
        # device constants made once per size (causal masks), least recently
        # used first; at most MAX_CONSTS are kept (a captured graph holds
        # its own references to the ones it reads)
        self._const = collections.OrderedDict()
        # (B, S, full_mask) -> captured last-token forward, least recently
        # used first; at most MAX_GRAPHS are kept
        self._graphs = collections.OrderedDict()
        self._generation = self.ws.generation
        self.trace = None  # list to record (site, inputs, outputs) of every qdc call
        self.trace_ptrs = []

    @classmethod
    def from_directory(cls, directory, device="cuda"):
        """QwenBackbone(dir; device) (src/backbone.jl:74-192).  BF16 checkpoint
        tensors are uploaded as their raw bits and widened on the device."""
        config, weights = load_weights(directory, raw_bf16=torch.device(device).type == "cuda")
        return cls(config, weights, device)

    @classmethod
    def random(cls, config, seed=0, device="cuda"):
        return cls(config, random_weights(config, seed, device=device), device)

    # ------------------------------------------------------------ helpers

    def rope(self, n):
        """Device cos/sin tables for positions 0..n-1 (src/backbone_cpu.jl:90-105)."""
        rows = max(int(n), 1)
        hit = self._rope.get(self.config.rotary_dim)
        if hit is None or hit[0].shape[0] < rows:
            hit = ops.rope_table(self.config.rope_theta, self.config.rotary_dim, rows,
                                 device=self.device)
            self._rope[self.config.rotary_dim] = hit
        return hit

    def _upper(self, n):
        """(n, n) bool, True strictly above the diagonal (made once per n)."""
        key = ("upper", n)
        t = self._const.get(key)
        if t is None:
            while len(self._const) >= MAX_CONSTS:
                self._const.popitem(last=False)
            t = self._const[key] = torch.ones((n, n), dtype=torch.bool, device=self.device).triu_(1)
        self._const.move_to_end(key)
        return t

    def _record(self, site, inputs, outputs):
        """With `trace` a list: append (site, inputs, outputs) of a qdc call
        (copies), and the outputs' device addresses to `trace_ptrs`."""
        if self.trace is not None:
            clone = lambda t: None if t is None else t.detach().clone()
            self.trace.append((site, tuple(clone(t) for t in inputs),
                               tuple(clone(t) for t in outputs)))
            self.trace_ptrs.append((site, tuple(t.data_ptr() for t in outputs if t is not None)))

    def forward_bytes(self, B, S, full_mask, host_mask=True, last_only=False):
        return forward_bytes(self.config, B, S, full_mask, host_mask, last_only)

    # ------------------------------------------------------ attention parts

    def _attend(self, s, q4, k4, v4, notallowed, m, Sq, S):
        """Causal GQA attention of m sequences (full_attention,
        src/backbone.jl:237-262; the CUDA extension's materialised form,
        ext/cuda_attention.jl:163-175): scores = q k^T * inv(sqrt(D)), keys
        not allowed at -floatmax (a query that sees none averages every
        key), softmax over keys, values = probs v.  q4 (m, Sq, Hq, D), k4 /
        v4 (m, S, Hkv, D) views; `notallowed` bool broadcastable to
        (m, Sq, S) or None.  Returns the (m, Hq, Sq, D) values slot."""
        cfg = self.config
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        G = Hq // Hkv
        qh, kh, vh = s["qh"][:m], s["kh"][:m], s["vh"][:m]
        qh.copy_(q4.permute(0, 2, 1, 3))
        kh.copy_(k4.permute(0, 2, 1, 3))
        vh.copy_(v4.permute(0, 2, 1, 3))
        # query heads of one kv head sit together (head h reads kv head h // G)
        scores, probs = s["scores"][:m * Hkv], s["probs"][:m * Hkv]
        torch.bmm(qh.view(m * Hkv, G * Sq, D), kh.view(m * Hkv, S, D).transpose(1, 2), out=scores)
        scores.mul_(float(np.float32(1) / np.sqrt(np.float32(D))))
        if notallowed is not None:
            scores.view(m, Hkv, G, Sq, S).masked_fill_(notallowed.view(-1, 1, 1, Sq, S), -FLOATMAX32)
        torch.ops.aten._softmax.out(scores, -1, False, out=probs)
        values = s["values"][:m]
        torch.bmm(probs, vh.view(m * Hkv, S, D), out=values.view(m * Hkv, G * Sq, D))
        return values

    def _full_attention(self, layer, y, B, S, masks):
        cfg = self.config
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        T = B * S
        s = self.ws.take_all(_full_spec(cfg, B, S))
        proj = torch.mm(y, layer["qkv"].t(), out=s["proj"])
        qw, kw = Hq * 2 * D, Hkv * D
        qgate = proj[:, :qw].view(T, Hq, 2 * D)
        k_raw = proj[:, qw:qw + kw].view(T, Hkv, D)
        v = proj[:, qw + kw:].view(T, Hkv, D)
        cos, sin = self.rope(S)
        q, k = ops.native_q_k_norm_rope(qgate[:, :, :D], k_raw, layer["q_norm"], layer["k_norm"],
                                        cfg.eps, cfg.rotary_dim, cos, sin, seq_len=S, q_out=s["q"],
                                        k_out=s["k"], ctx=self.ctx)
        self._record("q_norm_rope", (qgate[:, :, :D],), (q,))
        self._record("k_norm_rope", (k_raw,), (k,))
        gated = s["gated"]
        nb = s["qh"].shape[0]
        q4, k4, v4 = q.view(B, S, Hq, D), k.view(B, S, Hkv, D), v.view(B, S, Hkv, D)
        for b0 in range(0, B, nb):
            b1 = min(B, b0 + nb)
            na = masks["causal"] if masks["notallowed"] is None else masks["notallowed"][b0:b1]
            values = self._attend(s, q4[b0:b1], k4[b0:b1], v4[b0:b1], na, b1 - b0, S, S)
            rows = slice(b0 * S, b1 * S)
            ops.native_attn_gate(values, qgate[rows, :, D:], out=gated[rows], ctx=self.ctx)
            self._record("attn_gate", (values, qgate[rows, :, D:]), (gated[rows],))
        return torch.mm(gated, layer["out"].t(), out=s["out"])

    def _full_attention_last(self, layer, y, B, S, masks):
        """The final layer's attention for the last query of each sequence
        only: K/V over the whole context, Q of one token at position S-1
        (cpu_final_full_attention, src/backbone_cpu.jl:996-1041;
        last_token_layer, ext/cuda_attention.jl:190-269).  Returns (B, hidden)."""
        cfg = self.config
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        qw, kw = Hq * 2 * D, Hkv * D
        s = self.ws.take_all(_full_last_spec(cfg, B, S))
        y_last = y.view(B, S, -1)[:, S - 1]
        qgate = torch.mm(y_last, layer["qkv"][:qw].t(), out=s["qgate"]).view(B, Hq, 2 * D)
        kv = torch.mm(y, layer["qkv"][qw:].t(), out=s["kv"])
        k_raw = kv[:, :kw].view(B * S, Hkv, D)
        v = kv[:, kw:].view(B * S, Hkv, D)
        cos, sin = self.rope(S)
        q = ops.native_qk_norm_rope(qgate[:, :, :D], layer["q_norm"], cfg.eps, cfg.rotary_dim, cos, sin,
                                    pos_offset=S - 1, seq_len=1, out=s["q"], ctx=self.ctx)
        k = ops.native_qk_norm_rope(k_raw, layer["k_norm"], cfg.eps, cfg.rotary_dim, cos, sin,
                                    seq_len=S, out=s["k"], ctx=self.ctx)
        self._record("q_norm_rope_last", (qgate[:, :, :D],), (q,))
        self._record("k_norm_rope", (k_raw,), (k,))
        # the last query sees every key up to its own position: only the mask hides keys
        key_off = None if masks["key_off"] is None else masks["key_off"].view(B, 1, S)
        values = self._attend(s, q.view(B, 1, Hq, D), k.view(B, S, Hkv, D), v.view(B, S, Hkv, D),
                              key_off, B, 1, S)
        gated = ops.native_attn_gate(values, qgate[:, :, D:], out=s["gated"], ctx=self.ctx)
        self._record("attn_gate", (values, qgate[:, :, D:]), (gated,))
        return torch.mm(gated, layer["out"].t(), out=s["out"])

    def _delta_attention(self, layer, y, B, S, masks):
        cfg = self.config
        T = B * S
        C, vw = cfg.qkv_width, cfg.value_width
        s = self.ws.take_all(_delta_spec(cfg, B, S, masks["maskf"] is None))
        # masked tokens enter the DeltaNet as zeros (src/backbone.jl:286)
        masked = y if masks["maskf"] is None else torch.mul(y, masks["maskf"].view(T, 1), out=s["masked"])
        proj = torch.mm(masked, layer["proj"].t(), out=s["proj"])  # [qkv | z | a | b] per token
        # causal 4-tap conv + SiLU + q/k L2 norms in one qdc pass over the
        # projection (src/backbone.jl:287-314)
        q, k, v = ops.native_delta_conv_norm(proj, layer["conv"], cfg.key_heads, cfg.key_dim,
                                             cfg.value_heads, cfg.value_dim, seq_len=S, q_out=s["q"],
                                             k_out=s["k"], v_out=s["v"], ctx=self.ctx)
        self._record("delta_conv_norm", (proj[:, :C], layer["conv"]), (q, k, v))
        # beta = sigmoid(b), decay = a_decay * softplus(a + dt_bias), a and b
        # read in place from the projection (src/backbone.jl:292-297)
        beta, decay = ops.native_delta_gates(proj, C + vw, cfg.value_heads, layer["a_decay"],
                                             layer["dt_bias"], beta=s["beta"], decay=s["decay"],
                                             ctx=self.ctx)
        self._record("delta_gates", (proj[:, C + vw:C + vw + 2 * cfg.value_heads],), (beta, decay))
        o = chunked_delta(q.view(B, S, cfg.key_heads, cfg.key_dim), k.view(B, S, cfg.key_heads, cfg.key_dim),
                          v.view(B, S, cfg.value_heads, cfg.value_dim), beta.view(B, S, cfg.value_heads),
                          decay.view(B, S, cfg.value_heads), cfg.value_heads // cfg.key_heads, s, s["o"],
                          self._upper(DELTA_CHUNK), self._solve)
        o = o.view(T, cfg.value_heads, cfg.value_dim)
        z = proj[:, C:C + vw].view(T, cfg.value_heads, cfg.value_dim)
        gated = ops.native_gated_rms(o, z, layer["norm"], cfg.eps, out=s["gated"], ctx=self.ctx)
        self._record("gated_rms", (o, z), (gated,))
        return torch.mm(gated, layer["out"].t(), out=s["out"])

    def _solve(self, system, x):
        return ops.native_delta_solve(system, x, ctx=self.ctx)

    def _mlp(self, layer, y, rows):
        """native_mlp (src/backbone.jl:384-388): the [gate; up] GEMM, qdc
        SwiGLU, the down GEMM.  Returns the down projection slot."""
        I = self.config.intermediate
        s = self.ws.take_all(_mlp_spec(self.config, rows))
        gu = torch.mm(y, layer["gate_up"].t(), out=s["gate_up"])
        h, _ = ops.native_mlp_gate(gu[:, :I], gu[:, I:], out_f32=s["h"], ctx=self.ctx)
        self._record("swiglu", (gu[:, :I], gu[:, I:]), (h,))
        return torch.mm(h, layer["down"].t(), out=s["mlp"])

    def _masks(self, root, dmask, B, S, full_mask):
        """Device masks of one forward: keys a query may not see (causal and,
        unless every position is unmasked, the masked keys) and the float
        mask the DeltaNet input is multiplied by."""
        causal = self._upper(S).view(1, S, S) if "full_attention" in self.config.layer_types else None
        masks = {"causal": causal, "notallowed": None, "key_off": None, "maskf": None}
        if not full_mask:
            masks["maskf"] = root["maskf"]
            masks["maskf"].copy_(dmask)
            if causal is not None:
                key_off = torch.ne(dmask.view(B, S), 1, out=root["key_off"])
                masks["key_off"] = key_off
                masks["notallowed"] = torch.logical_or(causal, key_off.view(B, 1, S), out=root["notallowed"])
        return masks

    # -------------------------------------------------------------- forward

    def _forward(self, ids, mask, B, S, full_mask, last_only=False):
        """Final-normalized states: (B*S, hidden), or (B, hidden) for the
        last token of each sequence when `last_only` (the last-token forward
        of src/backbone.jl:390-396; its final full-attention layer runs one
        query and its MLP one token, as ext/cuda_workspace.jl:279-297
        does).  ids: host int32 array or int32 device tensor (B*S,); mask:
        host int array or int32 device tensor (B*S,); full_mask: whether
        every mask value is 1 (known on the host, so nothing here waits on
        the device).  The result is a workspace slot: valid until the
        model's next forward (callers hold the context lock and copy it
        out first)."""
        cfg = self.config
        ws = self.ws
        T, H = B * S, cfg.hidden
        host_mask = not torch.is_tensor(mask)
        ws.begin(forward_bytes(cfg, B, S, full_mask, host_mask, last_only))
        if ws.generation != self._generation:
            # the arena moved: graphs recorded against the old one are void
            self._graphs.clear()
            self._generation = ws.generation
        root = ws.take_all(_root_spec(cfg, B, S, full_mask, host_mask, "full_attention" in cfg.layer_types))
        if host_mask:
            dmask = root["mask"]
            dmask.copy_(torch.from_numpy(np.ascontiguousarray(np.asarray(mask).reshape(-1), np.int32)))
        else:
            dmask = mask
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            masks = self._masks(root, dmask, B, S, full_mask)
            layers = self.layers
            x, r, y = root["x"], root["r"], root["y"]
            ops.native_gather_rms(self.embedding, ids, layers[0]["input_norm"], cfg.eps, out_x=x, out_y=y,
                                  ctx=self.ctx)
            self._record("gather_rms", (), (x, y))
            for i, layer in enumerate(layers):
                last = i + 1 == len(layers)
                mark = ws.mark()
                if last and last_only:
                    return self._last_layer(layer, x, y, B, S, masks)
                if layer["kind"] == "full":
                    mixed = self._full_attention(layer, y, B, S, masks)
                else:
                    mixed = self._delta_attention(layer, y, B, S, masks)
                ops.native_residual_rms(x, mixed, layer["post_norm"], cfg.eps, out_r=r, out_y=y, ctx=self.ctx)
                self._record("post_rms", (x, mixed), (r, y))
                mlp = self._mlp(layer, y, T)
                nxt = self.final_norm if last else layers[i + 1]["input_norm"]
                r_in = r.clone() if self.trace is not None else None
                ops.native_residual_add_rms(r, mlp, nxt, cfg.eps, out_y=y, ctx=self.ctx)
                self._record("final_rms" if last else "mlp_rms", (r_in, mlp), (r, y))
                x, r = r, x
                ws.release(mark)
            return y
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev_tf32

    def _last_layer(self, layer, x, y, B, S, masks):
        """The final layer of the last-token forward: attention for the last
        query (full) or over every token (DeltaNet), then the post norm, MLP
        and final norm of the last token of each sequence.  The result goes
        to the first B rows of the root slot y."""
        cfg = self.config
        H = cfg.hidden
        rows = lambda t: t.view(B, S, H)[:, S - 1]  # the last token of each sequence
        if layer["kind"] == "full":
            mixed = self._full_attention_last(layer, y, B, S, masks)
        else:
            mixed = rows(self._delta_attention(layer, y, B, S, masks))
        r_last, y_last = self.ws.take((B, H)), self.ws.take((B, H))
        x_last = rows(x)
        ops.native_residual_rms(x_last, mixed, layer["post_norm"], cfg.eps, out_r=r_last, out_y=y_last,
                                ctx=self.ctx)
        self._record("post_rms", (x_last, mixed), (r_last, y_last))
        mlp = self._mlp(layer, y_last, B)
        r_in = r_last.clone() if self.trace is not None else None
        out = y[:B]
        ops.native_residual_add_rms(r_last, mlp, self.final_norm, cfg.eps, out_y=out, ctx=self.ctx)
        self._record("final_rms", (r_in, mlp), (r_last, out))
        return out

    def _hidden(self, ids, mask, last_only):
        """The forward of (B, S) host ids / mask; the caller holds ctx.lock.
        Returns the workspace slot of the result and (B, S)."""
        ids = np.asarray(ids)
        if ids.ndim != 2:
            raise ArgumentError(1, "batch_hidden takes (batch, sequence) ids")
        B, S = ids.shape
        mask = np.ones_like(ids) if mask is None else np.asarray(mask)
        if mask.shape != ids.shape:
            raise ArgumentError(1, "Input IDs and mask must have identical lengths.")
        check_sequence(self.config.vocab, ids.reshape(-1), mask.reshape(-1))
        y = self._forward(ids.reshape(-1).astype(np.int32), mask.reshape(-1), B, S,
                          bool((mask == 1).all()), last_only)
        self.ctx.sync()
        return y

    def batch_hidden(self, ids, mask=None, last_only=False, out=None):
        """Final-normalized states of B equal-length sequences on the device:
        (B*S, hidden), or (B, hidden) for each sequence's last token.
        ids / mask: (B, S) host arrays (mask default ones).  The result is
        copied out of the workspace into `out` (a new tensor when None)."""
        with self.ctx.lock:
            y = self._hidden(ids, mask, last_only)
            out = y.clone() if out is None else out.copy_(y)
            if out.is_cuda:  # the copy has left the workspace before another forward may reuse it
                torch.cuda.current_stream(out.device).synchronize()
            return out

    def host_hidden(self, ids, mask=None, last_only=False):
        """batch_hidden read back to a host float32 array inside the
        model's lock (no device allocation)."""
        with self.ctx.lock:
            return _host_copy(self._hidden(ids, mask, last_only))

    def last_hidden_graphed(self, ids, mask):
        """backbone_last_hidden through a CUDA graph cached per (batch,
        sequence, full mask): pinned host -> device copy of ids and mask,
        the forward on device ids, and the device -> pinned host copy of the
        result, replayed as one graph (ext/cuda_io_graph.jl:31-88).  Returns
        host (B, hidden).  A shape whose capture fails runs eagerly, as the
        reference falls back (ext/cuda_workspace.jl:247-252)."""
        ids = np.asarray(ids)
        mask = np.asarray(mask)
        if ids.ndim != 2 or mask.shape != ids.shape:
            raise ArgumentError(1, "Input IDs and mask must have identical lengths.")
        check_sequence(self.config.vocab, ids.reshape(-1), mask.reshape(-1))
        B, S = ids.shape
        key = (B, S, bool((mask == 1).all()))
        with self.ctx.lock:
            g = self._graphs.get(key)
            if g is not None and g.generation != self.ws.generation:
                g = None  # recorded against an arena that has since moved
            if g is None:
                while len(self._graphs) >= MAX_GRAPHS:
                    self._graphs.popitem(last=False)
                g = _GraphedLastHidden(self, *key)
                self._graphs[key] = g
            self._graphs.move_to_end(key)
            if g.graph is None:
                return _host_copy(self._hidden(ids, mask, True))
            return g(ids, mask)


def _host_copy(t):
    """A host numpy copy of workspace slot `t` (never a view of it)."""
    h = t.cpu()
    if h.data_ptr() == t.data_ptr():
        h = h.clone()
    return h.numpy()


class _GraphedLastHidden:
    """One captured last-token forward for a fixed (B, S, full_mask).  Its
    workspace slots are the model arena's, at the addresses of the capture;
    `generation` records which arena that was."""

    def __init__(self, model, B, S, full_mask):
        dev = model.device
        self.model = model
        self.ids_host = torch.zeros((B * S,), dtype=torch.int32).pin_memory()
        self.mask_host = torch.ones((B * S,), dtype=torch.int32).pin_memory()
        self.ids_dev = torch.zeros((B * S,), dtype=torch.int32, device=dev)
        self.mask_dev = torch.ones((B * S,), dtype=torch.int32, device=dev)
        self.out_host = torch.empty((B, model.config.hidden), dtype=torch.float32).pin_memory()
        self.stream = torch.cuda.Stream(dev)
        self.graph = None
        try:
            with torch.cuda.stream(self.stream):
                self._body(model, B, S, full_mask)  # warm-up: arena size, views, RoPE tables
            self.stream.synchronize()
            self.generation = model.ws.generation
            # the captured kernels read these tables by address: hold them, as
            # the model's cache replaces them when a longer sequence arrives
            self.rope = model.rope(S)
            self.consts = tuple(model._const.values())  # the masks the capture reads
            graph = torch.cuda.CUDAGraph()
            # thread_local: CUDA calls that other host threads make meanwhile
            # (outside this model's lock) do not invalidate the capture
            with torch.cuda.graph(graph, stream=self.stream, capture_error_mode="thread_local"):
                self._body(model, B, S, full_mask)
            if model.ws.generation == self.generation:
                self.graph = graph
        except RuntimeError:
            self.graph = None
            torch.cuda.synchronize(dev)
        self.generation = model.ws.generation

    def _body(self, model, B, S, full_mask):
        self.ids_dev.copy_(self.ids_host, non_blocking=True)
        self.mask_dev.copy_(self.mask_host, non_blocking=True)
        y = model._forward(self.ids_dev, self.mask_dev, B, S, full_mask, last_only=True)
        self.out_host.copy_(y, non_blocking=True)

    def __call__(self, ids, mask):
        self.ids_host.copy_(torch.from_numpy(np.ascontiguousarray(ids.reshape(-1), np.int32)))
        self.mask_host.copy_(torch.from_numpy(np.ascontiguousarray(mask.reshape(-1), np.int32)))
        # replay() launches on the current stream: make that the graph's own
        # stream, the one synchronised before the pinned output is read
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        self.stream.synchronize()
        self.model.ctx.sync(self.stream)
        return self.out_host.numpy().copy()


def chunked_delta(q, k, v, beta, decay, groups, slots, out, upper, solve, chunk=DELTA_CHUNK):
    """Gated delta rule in 64-token chunks (src/backbone.jl:309-343), batched
    over sequences, value heads and chunks; only the state hand-off between
    chunks is sequential.  Every intermediate is a slot of `slots`
    (_chunked_spec), written in place, so the rule allocates nothing.

    q, k: (B, S, Hk, Dk) normalised; v: (B, S, Hv, Dv); beta, decay: (B, S, Hv);
    value head h reads key head h // groups.  Writes o (B, S, Hv, Dv) into
    `out` and returns it.  A short last chunk is zero-padded: padded tokens
    have beta = 0, k = q = v = 0 and decay 0, so they change neither the
    real tokens' outputs nor the carried state.  `upper` is a (chunk, chunk)
    bool mask of the strict upper triangle; `solve(system, x)` solves
    x <- UnitLowerTriangular(system) \\ x in place for (N, chunk, chunk) /
    (N, chunk, width) batches (delta_solve, src/backbone.jl:279).

    The state hand-off runs as a linear scan when the slots hold "A"
    (few launches: latency-bound calls, batch x value heads <=
    SCAN_MAX_HEADS), else per chunk in the correction form (about half the
    arithmetic: throughput-bound calls)."""
    B, S, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    C = chunk
    n = -(-S // C)
    S2, P, W, BH = n * C, n * C - S, Dv + Dk, B * Hv
    N = BH * n
    g = slots
    Qh, Kh, Vh = g["Qh"], g["Kh"], g["Vh"]
    # head-major copies, padded to whole chunks
    for dst, src in ((Qh, q), (Kh, k)):
        d5 = dst.view(B, Hk, groups, S2, Dk)
        d5[:, :, :, :S].copy_(src.permute(0, 2, 1, 3).unsqueeze(2).expand(B, Hk, groups, S, Dk))
        if P:
            d5[:, :, :, S:].zero_()
    Vh[:, :, :S].copy_(v.permute(0, 2, 1, 3))
    bet, tail, cum = g["bet"], g["tail"], g["cum"]
    bet[:, :, :S].copy_(beta.permute(0, 2, 1))
    tail[:, :, :S].copy_(decay.permute(0, 2, 1))
    if P:
        for t in (Vh, bet, tail):
            t[:, :, S:].zero_()
    cum4 = cum.view(B, Hv, n, C)
    torch.cumsum(tail.view(B, Hv, n, C), -1, out=cum4)
    # pair[j, i] = exp(cum_j - cum_i) on and below the diagonal, 0 above
    # (never exp of a positive gap)
    pair = g["pair"]
    torch.sub(cum4.unsqueeze(-1), cum4.unsqueeze(-2), out=pair)
    pair.masked_fill_(upper, float("-inf"))
    torch.exp(pair, out=pair)
    Q3, K3, V3 = Qh.view(N, C, Dk), Kh.view(N, C, Dk), Vh.view(N, C, Dv)
    # system[i, j] = beta_i k_i.k_j pair[i, j]; the solve reads its strict lower triangle
    system = g["system"]
    torch.bmm(K3, K3.transpose(1, 2), out=system.view(N, C, C))
    system.mul_(bet.view(B, Hv, n, C, 1))
    system.mul_(pair)
    # one unit-lower-triangular solve for both right-hand sides
    # [V * beta | K * beta * exp(cum)] -> [new values | reading keys]
    e, be, X = g["e"], g["be"], g["X"]
    torch.exp(cum, out=e)
    torch.mul(bet, e, out=be)
    torch.mul(Vh.view(B, Hv, n, C, Dv), bet.view(B, Hv, n, C, 1), out=X[..., :Dv])
    torch.mul(Kh.view(B, Hv, n, C, Dk), be.view(B, Hv, n, C, 1), out=X[..., Dv:])
    solve(system.view(N, C, C), X.view(N, C, W))
    X3 = X.view(N, C, W)
    new_values, reading = X3[:, :, :Dv], X3[:, :, Dv:]
    intra = g["intra"]  # [j, i] = q_j k_i pair[j, i]
    torch.bmm(Q3, K3.transpose(1, 2), out=intra.view(N, C, C))
    intra.mul_(pair)
    qe = g["qe"]
    torch.mul(Qh.view(B, Hv, n, C, Dk), e.view(B, Hv, n, C, 1), out=qe)
    tail4 = tail.view(B, Hv, n, C)
    torch.sub(cum4[..., -1:], cum4, out=tail4)
    torch.exp(tail4, out=tail4)
    ending = g["ending"]  # E_c: keys decayed to the chunk's end
    torch.mul(Kh.view(B, Hv, n, C, Dk), tail4.unsqueeze(-1), out=ending)
    final = g["final"]  # f_c: the whole chunk's decay
    torch.exp(cum4[..., -1], out=final)
    U = g["U"]
    if "A" in g:
        # The hand-off is linear in the state S (Dv x Dk): with the chunk's
        # correction corr = new_values - reading @ S^T,
        #   S_c   = S_{c-1} f_c + corr^T E_c = S_{c-1} A_c + B_c,
        #           A_c = f_c I - reading^T E_c,  B_c = new_values^T E_c;
        #   out_c = qe S^T + intra corr = W_c S_{c-1}^T + U_c,
        #           W_c = qe - intra @ reading,   U_c = intra @ new_values.
        # A, B, W, U are batched over every chunk; the loop is one
        # multiply-add per chunk, and the outputs one batched product after.
        A, Bc, states = g["A"], g["Bc"], g["states"]
        torch.bmm(reading.transpose(1, 2), ending.view(N, C, Dk), out=A.view(N, Dk, Dk))
        A.neg_()
        A.diagonal(dim1=-2, dim2=-1).add_(final.view(B, Hv, n, 1))
        torch.bmm(new_values.transpose(1, 2), ending.view(N, C, Dk), out=Bc.view(N, Dv, Dk))
        qe.view(N, C, Dk).baddbmm_(intra.view(N, C, C), reading, alpha=-1)  # W in place of qe
        torch.bmm(intra.view(N, C, C), new_values, out=U.view(N, C, Dv))
        states[:, :, 0].zero_()  # states[:, :, c] = S_{c-1}
        for c in range(1, n):
            torch.baddbmm(Bc[:, :, c - 1].view(BH, Dv, Dk), states[:, :, c - 1].view(BH, Dv, Dk),
                          A[:, :, c - 1].view(BH, Dk, Dk), out=states[:, :, c].view(BH, Dv, Dk))
        U.view(N, C, Dv).baddbmm_(qe.view(N, C, Dk), states.view(N, Dv, Dk).transpose(1, 2))
    else:
        state, corr = g["state"], g["corr"]
        state.zero_()
        X5 = X.view(B, Hv, n, C, W)
        for c in range(n):
            nv = X5[:, :, c, :, :Dv].view(BH, C, Dv)
            rd = X5[:, :, c, :, Dv:].view(BH, C, Dk)
            torch.baddbmm(nv, rd, state.transpose(1, 2), alpha=-1, out=corr)   # new_values - reading S^T
            Uc = U[:, :, c].view(BH, C, Dv)
            torch.bmm(qe[:, :, c].view(BH, C, Dk), state.transpose(1, 2), out=Uc)  # qe S^T
            Uc.baddbmm_(intra[:, :, c].view(BH, C, C), corr)                       # + intra corr
            state.mul_(final[:, :, c].view(BH, 1, 1))
            state.baddbmm_(corr.transpose(1, 2), ending[:, :, c].view(BH, C, Dk))  # + corr^T E
    # token-major output, heads contiguous within a token (the layout the
    # gated norm reads)
    out.copy_(U.view(B, Hv, S2, Dv)[:, :, :S].permute(0, 2, 1, 3))
    return out


def backbone_hidden(backbone, ids, mask, positions=None):
    """src/backbone.jl:433-460: one sequence, returns host float32 (tokens,
    hidden) final-normalized states (all positions, or `positions`, 1-based
    as in the reference)."""
    ids = np.asarray(ids).reshape(-1) if np.ndim(ids) == 1 else np.asarray(ids)
    mask = np.asarray(mask)
    if ids.ndim == 2:
        if ids.shape[0] != 1 or mask.shape[0] != 1:
            raise ArgumentError(1, "Pass one sequence per call; batching is not implemented yet.")
        ids, mask = ids.reshape(-1), mask.reshape(-1)
    check_sequence(backbone.config.vocab, ids, mask)
    states = backbone.host_hidden(ids.reshape(1, -1), mask.reshape(1, -1))
    if positions is None:
        return states
    pos = np.asarray(positions)
    if pos.size and (pos.min() < 1 or pos.max() > states.shape[0]):
        raise ArgumentError(1, "Position is outside the sequence.")
    return states[pos - 1]


def backbone_last_hidden(backbone, ids, mask):
    """src/backbone.jl:470-490: the last position's state, host vector, by
    the last-token forward (one-query final attention layer, one-token final
    MLP) replayed as a cached CUDA graph; QDC_B200_GRAPH=0 runs it eagerly
    (the reference's QDC_CUDA_GRAPH switch, ext/cuda_workspace.jl:231)."""
    ids = np.asarray(ids).reshape(1, -1)
    mask = np.asarray(mask).reshape(1, -1)
    check_sequence(backbone.config.vocab, ids.reshape(-1), mask.reshape(-1))
    if os.environ.get("QDC_B200_GRAPH", "1") == "0":
        return backbone.host_hidden(ids, mask, last_only=True)[0]
    return backbone.last_hidden_graphed(ids, mask)[0]


def sequence_start(mask_row):
    """native_sequence_start with trimming on (src/backbone.jl:44-51): the
    0-based index of the first unmasked position, or the last position when
    every position is masked."""
    nz = np.flatnonzero(np.asarray(mask_row) != 0)
    return int(nz[0]) if nz.size else len(mask_row) - 1


def trim_padding_enabled():
    """The CUDA extension's padding switch (ext/QwenDecisionCoreCUDAExt.jl:
    12-20): complete sequences are kept unless QDC_B200_TRIM_PADDING=1 (the
    reference's QDC_CUDA_TRIM_PADDING), so timings compare like for like."""
    return os.environ.get("QDC_B200_TRIM_PADDING", "0") == "1"


def batch_backbone_hidden(backbone, ids, mask, trim_padding=None):
    """The batched hook of src/backbone.jl:66-70, as the reference's Metal
    extension implements it (ext/metal_batch_forward.jl:104-140): for
    (batch, seq) ids and mask, the final-normalized hidden state of each
    row's last position, host float32 (batch, hidden) -- Julia's
    (hidden, batch), one column per input row.

    Padding: like the reference's CUDA extension, complete sequences are
    kept by default (ext/QwenDecisionCoreCUDAExt.jl:12-20).  With
    `trim_padding=True` (or, when it is None, QDC_B200_TRIM_PADDING=1) the
    leading columns that are masked in every row are dropped first (the
    earliest native_sequence_start of the rows, src/backbone.jl:44-51); RoPE
    is relative and fully masked leading tokens add nothing to attention,
    the DeltaNet state or the conv, so trimming changes results by rounding
    only.  All rows go through one last-token forward, replayed as a cached
    CUDA graph per shape (QDC_B200_GRAPH=0: eagerly)."""
    ids = np.asarray(ids)
    mask = np.asarray(mask)
    if ids.ndim != 2 or mask.shape != ids.shape:
        raise ArgumentError(1, "batch_backbone_hidden takes (batch, sequence) ids and mask of one shape")
    for row in range(ids.shape[0]):
        check_sequence(backbone.config.vocab, ids[row], mask[row])
    if trim_padding is None:
        trim_padding = trim_padding_enabled()
    if trim_padding:
        first = min(sequence_start(m) for m in mask)
        ids, mask = np.ascontiguousarray(ids[:, first:]), np.ascontiguousarray(mask[:, first:])
    if os.environ.get("QDC_B200_GRAPH", "1") == "0":
        return backbone.host_hidden(ids, mask, last_only=True)
    return backbone.last_hidden_graphed(ids, mask)
