"""QwenBackbone on B200: the reference's forward with every per-layer row op
on libqdc_b200's sm_100a kernels.

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
                  causal GQA attention (torch SDPA), qdc sigmoid gate read
                  from the attention output in place, o GEMM;
                  delta: one [qkv;z;a;b] GEMM, qdc causal 4-tap conv + SiLU +
                  q/k L2 norms, qdc beta/decay gates, chunked gated delta
                  rule (torch), qdc gated norm reading z in place, out GEMM
  post norm    -- qdc residual add + RMSNorm
  MLP          -- one [gate;up] GEMM, qdc SwiGLU, down GEMM
  residual add -- fused with the next layer's input norm / the final norm.

The projections, attention, conv and delta rule are the reference's
out-of-scope parts; they run as plain torch Float32 ops (cuBLAS GEMMs with
TF32 disabled, as the reference computes in Float32, src/backbone.jl:14-16).
"""

import collections
import os

import numpy as np
import torch
import torch.nn.functional as F

from . import ops
from ._lib import ArgumentError
from .model import Config, device_f32, load_weights, pack_layers, random_weights

FLOATMAX32 = float(np.finfo(np.float32).max)
MAX_GRAPHS = 32  # cached last-token graphs per model (shapes beyond evict the oldest)
DELTA_CHUNK = 64  # src/backbone.jl:301, ext/cuda_delta_chunked.jl:9


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


class QwenBackbone:
    def __init__(self, config, weights, device="cuda"):
        self.config = config
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ArgumentError(1, "QwenBackbone(…; device) needs a CUDA device: the per-layer "
                                   "kernels have no CPU path")
        self.ctx = ops.context(self.device)
        self.embedding = _device_f32(weights["embed_tokens.weight"], self.device)
        self.final_norm = _device_f32(weights["norm.weight"], self.device)
        self.layers = pack_layers(config, weights, self.device)
        self._rope = {}
        # (B, S, full_mask) -> captured last-token forward, least recently
        # used first; at most MAX_GRAPHS are kept (each holds its own buffers)
        self._graphs = collections.OrderedDict()
        self.trace = None  # list to record (site, inputs, outputs) of every qdc call

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

    def _record(self, site, inputs, outputs):
        if self.trace is not None:
            clone = lambda t: None if t is None else t.detach().clone()
            self.trace.append((site, tuple(clone(t) for t in inputs),
                               tuple(clone(t) for t in outputs)))

    # ------------------------------------------------------ attention parts

    def _full_attention(self, layer, y, mask, B, S, full_mask):
        cfg = self.config
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        T = B * S
        proj = y @ layer["qkv"].t()
        qw, kw = Hq * 2 * D, Hkv * D
        qgate = proj[:, :qw].view(T, Hq, 2 * D)
        k_raw = proj[:, qw:qw + kw].view(T, Hkv, D)
        v = proj[:, qw + kw:].view(T, Hkv, D)
        cos, sin = self.rope(S)
        q, k = ops.native_q_k_norm_rope(qgate[:, :, :D], k_raw, layer["q_norm"], layer["k_norm"],
                                        cfg.eps, cfg.rotary_dim, cos, sin, seq_len=S, ctx=self.ctx)
        self._record("q_norm_rope", (qgate[:, :, :D],), (q,))
        self._record("k_norm_rope", (k_raw,), (k,))
        qh = q.view(B, S, Hq, D).transpose(1, 2)
        kh = k.view(B, S, Hkv, D).transpose(1, 2)
        vh = v.reshape(B, S, Hkv, D).transpose(1, 2)
        # key i visible to query j iff i <= j and mask[i] == 1, else -floatmax
        # (src/backbone.jl:237-242): a fully hidden query averages every key.
        if full_mask:
            out = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
        else:
            causal = torch.ones((S, S), dtype=torch.bool, device=self.device).tril()
            allowed = causal[None] & (mask.view(B, 1, S) == 1)
            bias = torch.zeros((B, 1, S, S), dtype=torch.float32, device=self.device)
            bias.masked_fill_(~allowed[:, None], -FLOATMAX32)
            out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=bias, enable_gqa=True)
        gated = ops.native_attn_gate(out, qgate[:, :, D:], ctx=self.ctx)
        self._record("attn_gate", (out, qgate[:, :, D:]), (gated,))
        return gated @ layer["out"].t()

    def _full_attention_last(self, layer, y, mask, B, S, full_mask):
        """The final layer's attention for the last query of each sequence
        only: K/V over the whole context, Q of one token at position S-1
        (cpu_final_full_attention, src/backbone_cpu.jl:996-1041;
        last_token_layer, ext/cuda_attention.jl:190-269).  Returns (B, hidden)."""
        cfg = self.config
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        qw, kw = Hq * 2 * D, Hkv * D
        y_last = y.view(B, S, -1)[:, S - 1]
        qgate = (y_last @ layer["qkv"][:qw].t()).view(B, Hq, 2 * D)
        kv = y @ layer["qkv"][qw:].t()
        k_raw = kv[:, :kw].view(B * S, Hkv, D)
        v = kv[:, kw:].view(B * S, Hkv, D)
        cos, sin = self.rope(S)
        q = ops.native_qk_norm_rope(qgate[:, :, :D], layer["q_norm"], cfg.eps, cfg.rotary_dim, cos, sin,
                                    pos_offset=S - 1, seq_len=1, ctx=self.ctx)
        k = ops.native_qk_norm_rope(k_raw, layer["k_norm"], cfg.eps, cfg.rotary_dim, cos, sin,
                                    seq_len=S, ctx=self.ctx)
        self._record("q_norm_rope_last", (qgate[:, :, :D],), (q,))
        self._record("k_norm_rope", (k_raw,), (k,))
        qh = q.view(B, 1, Hq, D).transpose(1, 2)
        kh = k.view(B, S, Hkv, D).transpose(1, 2)
        vh = v.reshape(B, S, Hkv, D).transpose(1, 2)
        if full_mask:  # the last query sees every key
            out = F.scaled_dot_product_attention(qh, kh, vh, enable_gqa=True)
        else:
            bias = torch.zeros((B, 1, 1, S), dtype=torch.float32, device=self.device)
            bias.masked_fill_(mask.view(B, 1, 1, S) != 1, -FLOATMAX32)
            out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=bias, enable_gqa=True)
        gated = ops.native_attn_gate(out, qgate[:, :, D:], ctx=self.ctx)
        self._record("attn_gate", (out, qgate[:, :, D:]), (gated,))
        return gated @ layer["out"].t()

    def _delta_attention(self, layer, y, mask, B, S, full_mask=False):
        cfg = self.config
        T = B * S
        kw, vw, C = cfg.key_width, cfg.value_width, cfg.qkv_width
        # masked tokens enter the DeltaNet as zeros (src/backbone.jl:286)
        masked = y if full_mask else y * mask.view(T, 1).to(torch.float32)
        proj = masked @ layer["proj"].t()  # [qkv | z | a | b] per token
        # causal 4-tap conv + SiLU + q/k L2 norms in one qdc pass over the
        # projection (src/backbone.jl:287-314)
        q, k, v = ops.native_delta_conv_norm(proj, layer["conv"], cfg.key_heads, cfg.key_dim,
                                             cfg.value_heads, cfg.value_dim, seq_len=S, ctx=self.ctx)
        self._record("delta_conv_norm", (proj[:, :C], layer["conv"]), (q, k, v))
        q = q.view(B, S, cfg.key_heads, cfg.key_dim)
        k = k.view(B, S, cfg.key_heads, cfg.key_dim)
        v = v.view(B, S, cfg.value_heads, cfg.value_dim)
        # beta = sigmoid(b), decay = a_decay * softplus(a + dt_bias), a and b
        # read in place from the projection (src/backbone.jl:292-297)
        beta, decay = ops.native_delta_gates(proj, C + vw, cfg.value_heads, layer["a_decay"],
                                             layer["dt_bias"], ctx=self.ctx)
        self._record("delta_gates", (proj[:, C + vw:C + vw + 2 * cfg.value_heads],), (beta, decay))
        beta = beta.view(B, S, cfg.value_heads)
        decay = decay.view(B, S, cfg.value_heads)
        o = chunked_delta(q, k, v, beta, decay, cfg.value_heads // cfg.key_heads)
        o = o.reshape(T, cfg.value_heads, cfg.value_dim)
        z = proj[:, C:C + vw].view(T, cfg.value_heads, cfg.value_dim)
        gated = ops.native_gated_rms(o, z, layer["norm"], cfg.eps, ctx=self.ctx)
        self._record("gated_rms", (o, z), (gated,))
        return gated @ layer["out"].t()

    # -------------------------------------------------------------- forward

    def _forward(self, ids, mask, B, S, full_mask, last_only=False):
        """Final-normalized states on the device: (B*S, hidden), or (B, hidden)
        for the last token of each sequence when `last_only` (the last-token
        forward of src/backbone.jl:390-396; its final full-attention layer runs
        one query and its MLP one token, as ext/cuda_workspace.jl:279-297
        does).  ids: host int32 array or int32 device tensor (B*S,); mask:
        int device tensor (B*S,); full_mask: whether every mask value is 1
        (known on the host, so nothing here waits on the device)."""
        cfg = self.config
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            layers = self.layers
            x, y = ops.native_gather_rms(self.embedding, ids, layers[0]["input_norm"], cfg.eps,
                                         ctx=self.ctx)
            self._record("gather_rms", (), (x, y))
            I = cfg.intermediate
            for i, layer in enumerate(layers):
                last = i + 1 == len(layers)
                if last and last_only:
                    rows = lambda t: t.view(B, S, -1)[:, S - 1]  # the last token of each sequence
                    if layer["kind"] == "full":
                        mixed = self._full_attention_last(layer, y, mask, B, S, full_mask)
                    else:
                        mixed = rows(self._delta_attention(layer, y, mask, B, S, full_mask))
                    x = rows(x)
                elif layer["kind"] == "full":
                    mixed = self._full_attention(layer, y, mask, B, S, full_mask)
                else:
                    mixed = self._delta_attention(layer, y, mask, B, S, full_mask)
                r, y = ops.native_residual_rms(x, mixed, layer["post_norm"], cfg.eps, ctx=self.ctx)
                self._record("post_rms", (x, mixed), (r, y))
                gu = y @ layer["gate_up"].t()
                h, _ = ops.native_mlp_gate(gu[:, :I], gu[:, I:], ctx=self.ctx)
                self._record("swiglu", (gu[:, :I], gu[:, I:]), (h,))
                mlp = h @ layer["down"].t()
                nxt = self.final_norm if last else layers[i + 1]["input_norm"]
                r_in = r.clone() if self.trace is not None else None
                x, y = ops.native_residual_add_rms(r, mlp, nxt, cfg.eps, ctx=self.ctx)
                self._record("final_rms" if last else "mlp_rms", (r_in, mlp), (x, y))
            return y
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev_tf32

    def batch_hidden(self, ids, mask=None, last_only=False):
        """Final-normalized states of B equal-length sequences on the device:
        (B*S, hidden), or (B, hidden) for each sequence's last token.
        ids / mask: (B, S) host arrays (mask default ones)."""
        ids = np.asarray(ids)
        if ids.ndim != 2:
            raise ArgumentError(1, "batch_hidden takes (batch, sequence) ids")
        B, S = ids.shape
        mask = np.ones_like(ids) if mask is None else np.asarray(mask)
        if mask.shape != ids.shape:
            raise ArgumentError(1, "Input IDs and mask must have identical lengths.")
        check_sequence(self.config.vocab, ids.reshape(-1), mask.reshape(-1))
        dmask = torch.from_numpy(mask.reshape(-1).astype(np.int32)).to(self.device)
        with self.ctx.lock:
            y = self._forward(ids.reshape(-1).astype(np.int32), dmask, B, S,
                              bool((mask == 1).all()), last_only)
            self.ctx.sync()
        return y

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
            if g is None:
                while len(self._graphs) >= MAX_GRAPHS:
                    self._graphs.popitem(last=False)
                g = self._graphs[key] = _GraphedLastHidden(self, *key)
            self._graphs.move_to_end(key)
            if g.graph is None:
                return self.batch_hidden(ids, mask, last_only=True).cpu().numpy()
            return g(ids, mask)


class _GraphedLastHidden:
    """One captured last-token forward for a fixed (B, S, full_mask)."""

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
                self._body(model, B, S, full_mask)  # warm-up: lazy handles, RoPE tables
            self.stream.synchronize()
            # the captured kernels read these tables by address: hold them, as
            # the model's cache replaces them when a longer sequence arrives
            self.rope = model.rope(S)
            graph = torch.cuda.CUDAGraph()
            # thread_local: CUDA calls that other host threads make meanwhile
            # (outside this model's lock) do not invalidate the capture
            with torch.cuda.graph(graph, stream=self.stream, capture_error_mode="thread_local"):
                self._body(model, B, S, full_mask)
            self.graph = graph
        except RuntimeError:
            self.graph = None
            torch.cuda.synchronize(dev)

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
    states = backbone.batch_hidden(ids.reshape(1, -1), mask.reshape(1, -1)).cpu().numpy()
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
        return backbone.batch_hidden(ids, mask, last_only=True).cpu().numpy()[0]
    return backbone.last_hidden_graphed(ids, mask)[0]


SCAN_MAX_HEADS = 64  # batch x value heads up to which the hand-off runs as a linear scan


def chunked_delta(q, k, v, beta, decay, groups, chunk=DELTA_CHUNK, scan=None):
    """Gated delta rule in 64-token chunks (src/backbone.jl:309-343), batched
    over sequences, value heads and chunks; only the state hand-off between
    chunks is sequential.

    q, k: (B, S, Hk, Dk) normalised; v: (B, S, Hv, Dv); beta, decay: (B, S, Hv).
    Returns o: (B, S, Hv, Dv).  A short last chunk is zero-padded: padded
    tokens have beta = 0, k = q = v = 0 and decay 0, so they change neither
    the real tokens' outputs nor the carried state.

    `scan` picks how the hand-off runs: as a linear recurrence in the state,
    one batched multiply-add per chunk (few launches: latency-bound calls,
    batch x value heads <= SCAN_MAX_HEADS by default), or per chunk in the
    correction form (about half the arithmetic: throughput-bound calls)."""
    B, S, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    n = (S + chunk - 1) // chunk
    P = n * chunk - S
    idx = torch.arange(Hv, device=q.device) // groups  # kv head of value head h: cld(h, groups)

    def per_head(t, heads_idx=None):  # (B, S, H, D) -> (B, H, n, C, D)
        if heads_idx is not None and groups > 1:
            t = t[:, :, heads_idx]
        if P:
            t = F.pad(t, (0, 0, 0, 0, 0, P))
        return t.view(B, n, chunk, t.shape[2], t.shape[3]).permute(0, 3, 1, 2, 4)

    def per_head_scalar(t):  # (B, S, H) -> (B, H, n, C)
        if P:
            t = F.pad(t, (0, 0, 0, P))
        return t.view(B, n, chunk, Hv).permute(0, 3, 1, 2)

    Q, K, V = per_head(q, idx), per_head(k, idx), per_head(v)
    bet = per_head_scalar(beta)
    cum = torch.cumsum(per_head_scalar(decay), dim=-1)
    upper = torch.ones((chunk, chunk), dtype=torch.bool, device=q.device).triu(1)
    diff = cum[..., :, None] - cum[..., None, :]
    # exp(cum_j - cum_i) on and below the diagonal, 0 above (never exp of a positive gap)
    pair = torch.exp(diff.masked_fill_(upper, float("-inf")))                  # (B,H,n,C,C)
    kb = K * bet[..., None]
    system = (kb @ K.transpose(-1, -2)) * pair
    L = torch.tril(system, diagonal=-1) + torch.eye(chunk, device=q.device)
    e = torch.exp(cum)[..., None]
    # one unit-lower-triangular solve for both right-hand sides
    both = torch.linalg.solve_triangular(L, torch.cat([V * bet[..., None], kb * e], dim=-1),
                                         upper=False, unitriangular=True)
    new_values, reading = both[..., :Dv], both[..., Dv:]
    intra_t = (Q @ K.transpose(-1, -2)) * pair                                  # [j, i] = q_j k_i pair[j,i]
    qe = Q * e
    end = cum[..., -1:]
    ending = K * torch.exp(end - cum)[..., None]                                # E_c: (B,H,n,C,Dk)
    final = torch.exp(end)[..., None]                                           # f_c: (B,H,n,1,1)
    if scan is None:
        scan = B * Hv <= SCAN_MAX_HEADS
    if not scan:
        state = torch.zeros((B, Hv, Dv, Dk), dtype=q.dtype, device=q.device)
        out = torch.empty((B, n, chunk, Hv, Dv), dtype=q.dtype, device=q.device)
        for c in range(n):
            corr = new_values[:, :, c] - reading[:, :, c] @ state.transpose(-1, -2)  # (B,H,C,Dv)
            out[:, c] = (qe[:, :, c] @ state.transpose(-1, -2) + intra_t[:, :, c] @ corr).transpose(1, 2)
            state = state * final[:, :, c] + corr.transpose(-1, -2) @ ending[:, :, c]
        out = out.view(B, n * chunk, Hv, Dv)
        return out if P == 0 else out[:, :S].contiguous()
    # The hand-off is linear in the state S (Dv x Dk): with the chunk's
    # correction corr = new_values - reading @ S^T,
    #   S_c   = S_{c-1} f_c + corr^T E_c = S_{c-1} A_c + B_c,
    #           A_c = f_c I - reading^T E_c,  B_c = new_values^T E_c;
    #   out_c = qe S^T + intra corr = W_c S_{c-1}^T + U_c,
    #           W_c = qe - intra @ reading,   U_c = intra @ new_values.
    # A, B, W, U are batched over every chunk; the loop is one multiply-add
    # per chunk, and the outputs are one batched product afterwards.
    eye = torch.eye(Dk, dtype=q.dtype, device=q.device)
    chunk_major = lambda t: t.permute(2, 0, 1, 3, 4).reshape(n, B * Hv, t.shape[-2], t.shape[-1])
    A = chunk_major(final * eye - reading.transpose(-1, -2) @ ending)           # (n,BH,Dk,Dk)
    Bc = chunk_major(new_values.transpose(-1, -2) @ ending)                     # (n,BH,Dv,Dk)
    W = qe - intra_t @ reading                                                  # (B,H,n,C,Dk)
    U = intra_t @ new_values                                                    # (B,H,n,C,Dv)
    states = torch.empty((n + 1, B * Hv, Dv, Dk), dtype=q.dtype, device=q.device)  # S_0 .. S_n
    states[0].zero_()
    for c in range(n):
        torch.baddbmm(Bc[c], states[c], A[c], out=states[c + 1])
    before = states[:n].view(n, B, Hv, Dv, Dk).permute(1, 2, 0, 3, 4)            # S_{c-1}: (B,H,n,Dv,Dk)
    # token-major output, heads contiguous within a token (the layout the
    # gated norm reads)
    out = (W @ before.transpose(-1, -2) + U).permute(0, 2, 3, 1, 4).contiguous()  # (B,n,C,H,Dv)
    out = out.view(B, n * chunk, Hv, Dv)
    return out if P == 0 else out[:, :S].contiguous()


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
        return backbone.batch_hidden(ids, mask, last_only=True).cpu().numpy()
    return backbone.last_hidden_graphed(ids, mask)
