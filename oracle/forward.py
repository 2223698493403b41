"""Whole-forward CPU restatement of QwenDecisionCore.jl's `backbone_hidden`.

TEST INFRASTRUCTURE ONLY.  It exists to pin the oracle's per-layer ops
(oracle/qdc_oracle.c) against the reference's golden logits
(test/fixtures/native/reference.json, checked at 2e-5 by the reference's
test/backbone.jl:1-34): every norm / RoPE / gate / SwiGLU site of the
forward runs through the C oracle, as does the DeltaNet prologue (4-tap
causal conv + SiLU + q/k L2 norms); the out-of-scope parts (projections,
causal attention and the gated delta rule) run in float64 numpy.

Reference call stack restated here (src/backbone.jl):
  backbone_hidden :433-460 -> native_gather :55-64 -> native_hidden_states
  :406-411 -> native_layer :363-367 (input RMSNorm, attention,
  native_residual_rms :347-350, native_mlp :384-388 with the SwiGLU gate
  :352-355, native_residual_add! :358-361) -> final RMSNorm :410.
  full_attention :224-262 (q/k norm + partial RoPE in the CPU form of
  src/backbone_cpu.jl:90-136), delta_attention :284-345 (the chunked rule
  is restated in its equivalent token-recurrent form, src/backbone_cpu.jl:
  681-705 and :744-756, in float64).

Weights are kept in safetensors / torch orientation, (out, in) row-major;
the reference reverses axes on load (src/safetensors.jl:1-3,14), so its
`transpose(W) * x` is `x @ W.T` here with x of shape (tokens, hidden).
"""
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from . import oracle as O

FLOATMAX32 = float(np.finfo(np.float32).max)


# --- safetensors reader, src/safetensors.jl:3-35 -----------------------------

def read_safetensors(path):
    """Row-major tensors as numpy float32 (BF16 decoded by bits << 16)."""
    out = {}
    with open(path, "rb") as f:
        raw = f.read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    if not 0 < hlen <= len(raw) - 8:
        raise ValueError("Invalid safetensors header.")
    header = json.loads(raw[8:8 + hlen])
    base = 8 + hlen
    for name, spec in header.items():
        if name == "__metadata__":
            continue
        start, stop = spec["data_offsets"]
        shape = tuple(spec["shape"])
        blob = raw[base + start: base + stop]
        if spec["dtype"] == "F32":
            arr = np.frombuffer(blob, "<f4").astype(np.float32)
        elif spec["dtype"] == "F16":
            arr = np.frombuffer(blob, "<f2").astype(np.float32)
        elif spec["dtype"] == "BF16":
            arr = (np.frombuffer(blob, "<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError("unsupported dtype " + spec["dtype"])
        out[name] = arr.reshape(shape)
    return out


# --- model -----------------------------------------------------------------

@dataclass
class Config:
    """Fields of the reference's `config` NamedTuple, src/backbone.jl:90-102."""
    hidden: int
    head_dim: int
    heads: int
    kv_heads: int
    key_heads: int
    value_heads: int
    key_dim: int
    value_dim: int
    eps: float
    rope_theta: float
    rotary_dim: int
    vocab: int = 0
    intermediate: int = 0
    conv_kernel: int = 4
    layer_types: list = field(default_factory=list)


@dataclass
class Model:
    config: Config
    weights: dict  # canonical name (without "language_model.") -> float32 array


def config_from_json(source):
    cfg = source["text_config"]
    rope = cfg["rope_parameters"]
    return Config(
        hidden=int(cfg["hidden_size"]), head_dim=int(cfg["head_dim"]),
        heads=int(cfg["num_attention_heads"]), kv_heads=int(cfg["num_key_value_heads"]),
        key_heads=int(cfg["linear_num_key_heads"]),
        value_heads=int(cfg["linear_num_value_heads"]),
        key_dim=int(cfg["linear_key_head_dim"]), value_dim=int(cfg["linear_value_head_dim"]),
        eps=float(np.float32(cfg["rms_norm_eps"])),
        rope_theta=float(np.float32(rope["rope_theta"])),
        # head_dim * rope_parameters.partial_rotary_factor, src/backbone.jl:101
        rotary_dim=int(cfg["head_dim"] * rope["partial_rotary_factor"]),
        vocab=int(cfg["vocab_size"]), intermediate=int(cfg["intermediate_size"]),
        conv_kernel=int(cfg.get("linear_conv_kernel_dim", 4)),
        layer_types=list(cfg["layer_types"]),
    )


def load_model(directory):
    with open(os.path.join(directory, "config.json")) as f:
        config = config_from_json(json.load(f))
    raw = read_safetensors(os.path.join(directory, "model.safetensors"))
    weights = {}
    for name, value in raw.items():
        at = name.find("language_model.")
        if at >= 0:
            weights[name[at + len("language_model."):]] = value
    return Model(config, weights)


def random_model(cfg, seed=0, std=0.02, gated_gamma_one=True):
    """Seeded random-init weights of a Qwen3.5-style hybrid backbone.

    Linear weights N(0, std); zero-centred norm gammas N(0, std) (applied as
    1+w); the DeltaNet output-norm gamma 1 + N(0, std) (applied as w,
    src/backbone.jl:339); A_log, dt_bias small; conv N(0, std)."""
    rng = np.random.default_rng(seed)
    H, I = cfg.hidden, cfg.intermediate
    n = lambda *shape: rng.normal(0.0, std, size=shape).astype(np.float32)
    w = {"embed_tokens.weight": n(cfg.vocab, H), "norm.weight": n(H)}
    kw = cfg.key_heads * cfg.key_dim
    vw = cfg.value_heads * cfg.value_dim
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        w[p + "input_layernorm.weight"] = n(H)
        w[p + "post_attention_layernorm.weight"] = n(H)
        w[p + "mlp.gate_proj.weight"] = n(I, H)
        w[p + "mlp.up_proj.weight"] = n(I, H)
        w[p + "mlp.down_proj.weight"] = n(H, I)
        if kind == "full_attention":
            D = cfg.head_dim
            w[p + "self_attn.q_proj.weight"] = n(2 * D * cfg.heads, H)
            w[p + "self_attn.k_proj.weight"] = n(D * cfg.kv_heads, H)
            w[p + "self_attn.v_proj.weight"] = n(D * cfg.kv_heads, H)
            w[p + "self_attn.o_proj.weight"] = n(H, D * cfg.heads)
            w[p + "self_attn.q_norm.weight"] = n(D)
            w[p + "self_attn.k_norm.weight"] = n(D)
        else:
            C = 2 * kw + vw
            w[p + "linear_attn.in_proj_qkv.weight"] = n(C, H)
            w[p + "linear_attn.in_proj_z.weight"] = n(vw, H)
            w[p + "linear_attn.in_proj_a.weight"] = n(cfg.value_heads, H)
            w[p + "linear_attn.in_proj_b.weight"] = n(cfg.value_heads, H)
            w[p + "linear_attn.conv1d.weight"] = n(C, 1, cfg.conv_kernel)
            w[p + "linear_attn.A_log"] = rng.uniform(-1.0, 0.5, cfg.value_heads).astype(np.float32)
            w[p + "linear_attn.dt_bias"] = n(cfg.value_heads)
            g = n(cfg.value_dim)
            w[p + "linear_attn.norm.weight"] = (1.0 + g).astype(np.float32) if gated_gamma_one else g
            w[p + "linear_attn.out_proj.weight"] = n(H, vw)
    return Model(cfg, w)


# --- out-of-scope parts, float64 --------------------------------------------

def _linear(W, x):
    return np.asarray(x, np.float64) @ np.asarray(W, np.float64).T


def full_attention(w, p, x, mask, cfg, trace=None):
    """src/backbone.jl:224-262 with the CPU q/k norm + RoPE of
    src/backbone_cpu.jl:113-136 (tables :90-105) through the oracle."""
    T = x.shape[0]
    D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    qgate = _linear(w[p + "self_attn.q_proj.weight"], x).astype(np.float32).reshape(T, Hq, 2 * D)
    cos, sin = O.rope_table(cfg.rope_theta, cfg.rotary_dim, max(T, 1))
    q = O.qk_norm_rope(qgate[:, :, :D], w[p + "self_attn.q_norm.weight"], cfg.eps,
                       cfg.rotary_dim, cos, sin)
    k_raw = _linear(w[p + "self_attn.k_proj.weight"], x).astype(np.float32).reshape(T, Hkv, D)
    k = O.qk_norm_rope(k_raw, w[p + "self_attn.k_norm.weight"], cfg.eps, cfg.rotary_dim, cos, sin)
    if trace is not None:
        trace.append(("q_norm_rope", p, qgate, q))
        trace.append(("k_norm_rope", p, k_raw, k))
    v = _linear(w[p + "self_attn.v_proj.weight"], x).reshape(T, Hkv, D)
    # key i visible to query j iff i <= j and mask[i] == 1, else -floatmax
    i = np.arange(T)[:, None]
    j = np.arange(T)[None, :]
    allowed = (i <= j) & (np.asarray(mask)[:, None] == 1)
    bias = np.where(allowed, 0.0, -FLOATMAX32)
    groups = Hq // Hkv
    values = np.empty((1, Hq, T, D), np.float32)
    for h in range(Hq):
        kv = h // groups
        scores = (k[:, kv, :].astype(np.float64) @ q[:, h, :].astype(np.float64).T) / np.sqrt(D)
        scores = scores + bias  # (keys, queries)
        probs = np.exp(scores - scores.max(axis=0, keepdims=True))
        probs /= probs.sum(axis=0, keepdims=True)
        values[0, h] = (probs.T @ v[:, kv, :]).astype(np.float32)  # (queries, D)
    # values .* native_sigmoid.(gate) through the oracle (src/backbone.jl:258-259)
    out = O.attn_gate(values, qgate[:, :, D:])
    if trace is not None:
        trace.append(("attn_gate", p, (values, qgate[:, :, D:]), out))
    return _linear(w[p + "self_attn.o_proj.weight"], out)


def delta_attention(w, p, x, mask, cfg, trace=None):
    """src/backbone.jl:284-345 (gated delta rule, token-recurrent form of
    src/backbone_cpu.jl:681-705) with the gated RMSNorm through the oracle."""
    T = x.shape[0]
    kw = cfg.key_dim * cfg.key_heads
    masked = np.asarray(x, np.float64) * np.asarray(mask, np.float64)[:, None]
    qkv = _linear(w[p + "linear_attn.in_proj_qkv.weight"], masked).astype(np.float32)
    conv = w[p + "linear_attn.conv1d.weight"]
    # causal 4-tap conv + SiLU + q/k L2 norms through the oracle
    # (src/backbone_cpu.jl:787-807, :411-427; generic src/backbone.jl:287-314)
    q, k, v = O.delta_conv_norm(qkv, conv.reshape(conv.shape[0], conv.shape[-1]), cfg.key_heads,
                                cfg.key_dim, cfg.value_heads, cfg.value_dim, seq_len=T)
    if trace is not None:
        trace.append(("delta_conv_norm", p, qkv, (q, k, v)))
    q, k, v = q.astype(np.float64), k.astype(np.float64), v.astype(np.float64)
    z = _linear(w[p + "linear_attn.in_proj_z.weight"], masked).astype(np.float32)
    z = z.reshape(T, cfg.value_heads, cfg.value_dim)
    # beta = sigmoid(b), decay = a_decay * softplus(a + dt_bias) through the
    # oracle on Float32 projections (src/backbone.jl:292-297); a_decay =
    # -1 * exp(A_log) in Float32 (src/backbone.jl:162)
    ab = np.concatenate([_linear(w[p + "linear_attn.in_proj_a.weight"], masked),
                         _linear(w[p + "linear_attn.in_proj_b.weight"], masked)], axis=1)
    ab = ab.astype(np.float32)
    a_decay = -np.exp(w[p + "linear_attn.A_log"].astype(np.float32))
    beta, decay = O.delta_gates(ab, 0, cfg.value_heads, a_decay, w[p + "linear_attn.dt_bias"])
    if trace is not None:
        trace.append(("delta_gates", p, ab, (beta, decay)))
    beta, decay = beta.astype(np.float64), decay.astype(np.float64)
    groups = cfg.value_heads // cfg.key_heads
    result = np.empty((T, cfg.value_heads, cfg.value_dim))
    for h in range(cfg.value_heads):
        kh = h // groups
        qh, kk = q[:, kh, :], k[:, kh, :]  # normalised by delta_conv_norm
        state = np.zeros((cfg.value_dim, cfg.key_dim))
        for t in range(T):
            f = np.exp(decay[t, h])
            projected = beta[t, h] * (v[t, h] - f * (state @ kk[t]))
            state = f * state + np.outer(projected, kk[t])
            result[t, h] = state @ qh[t]
    o = result.astype(np.float32)
    gated = O.gated_rms(o, z, w[p + "linear_attn.norm.weight"], cfg.eps)
    if trace is not None:
        trace.append(("gated_rms", p, (o, z), gated))
    return _linear(w[p + "linear_attn.out_proj.weight"], gated)


# --- backbone_hidden, src/backbone.jl:433-460 ---------------------------------

def check_sequence(model, ids, mask):
    """src/backbone.jl:413-422."""
    if len(ids) != len(mask):
        raise ValueError("Input IDs and mask must have identical lengths.")
    if len(ids) == 0:
        raise ValueError("Inputs must not be empty.")
    vocab = model.weights["embed_tokens.weight"].shape[0]
    if not all(0 <= int(i) < vocab for i in ids):
        raise ValueError("Token ID is outside the vocabulary.")
    if not all(int(m) in (0, 1) for m in mask):
        raise ValueError("Mask values must be zero or one.")


def backbone_hidden(model, ids, mask, trace=None):
    """Final-normalized hidden states, shape (tokens, hidden) float32."""
    check_sequence(model, ids, mask)
    cfg, w = model.config, model.weights
    hidden = O.gather(w["embed_tokens.weight"], np.asarray(ids, np.int32))
    for idx, kind in enumerate(cfg.layer_types):
        p = f"layers.{idx}."
        normalized = O.rms(hidden, w[p + "input_layernorm.weight"], cfg.eps)
        if trace is not None:
            trace.append(("input_rms", p, hidden, normalized))
        if kind == "full_attention":
            mixed = full_attention(w, p, normalized, mask, cfg, trace)
        else:
            mixed = delta_attention(w, p, normalized, mask, cfg, trace)
        mixed = mixed.astype(np.float32)
        residual, normalized = O.residual_rms(hidden, mixed, w[p + "post_attention_layernorm.weight"],
                                              cfg.eps)
        if trace is not None:
            trace.append(("post_rms", p, (hidden, mixed), (residual, normalized)))
        gate = _linear(w[p + "mlp.gate_proj.weight"], normalized).astype(np.float32)
        up = _linear(w[p + "mlp.up_proj.weight"], normalized).astype(np.float32)
        h, _ = O.swiglu(gate, up)
        if trace is not None:
            trace.append(("swiglu", p, (gate, up), h))
        mlp = _linear(w[p + "mlp.down_proj.weight"], h).astype(np.float32)
        hidden = (residual + mlp).astype(np.float32)  # native_residual_add!
    out = O.rms(hidden, w["norm.weight"], cfg.eps)
    if trace is not None:
        trace.append(("final_rms", "", hidden, out))
    return out


def probe_logits(model, readout, ids_rows, mask_rows):
    """The reference test's stand-in linear head, test/runtests.jl:23-31."""
    out = []
    for ids, mask in zip(ids_rows, mask_rows):
        states = backbone_hidden(model, ids, mask)
        out.append(readout.astype(np.float64) @ states[-1].astype(np.float64))
    return np.array(out)
