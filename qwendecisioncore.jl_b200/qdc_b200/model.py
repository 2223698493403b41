"""Model description, weight loading and packing for the B200 backbone.

  Config                  the reference's config NamedTuple, src/backbone.jl:90-102
  read_safetensors        src/safetensors.jl:3-35 (BF16 decoded as bits << 16)
  load_weights            QwenBackbone's weight selection and canonical names,
                          src/backbone.jl:107-135
  pack_layers             one projection GEMM per block, as the reference's
                          CUDA extension packs them (ext/cuda_mlp.jl:9-47):
                          [q; k; v], [qkv; z; a; b], [gate; up]
  random_weights          seeded random-init weights of a given shape

Weights stay in safetensors / torch orientation (out, in): the reference
reverses axes on load (src/safetensors.jl:1-3), so its `transpose(W) * x` is
`x @ W.T` on (tokens, hidden) activations here.
"""
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

QWEN_BACKBONE_TYPES = ("qwen3_5", "qwen3_5_text", "qwen3_8", "qwen3_8_text")  # src/backbone.jl:72


@dataclass
class Config:
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
    vocab: int
    intermediate: int
    conv_kernel: int = 4
    layer_types: list = field(default_factory=list)

    @classmethod
    def from_json(cls, source):
        """src/backbone.jl:78-106, with its validation."""
        if source.get("model_type") not in QWEN_BACKBONE_TYPES:
            raise ValueError("QwenBackbone supports Qwen3.5 / Qwen3.8 text backbones, got "
                             f"{source.get('model_type')}.")
        cfg = source["text_config"]
        if cfg.get("attention_bias", False):
            raise ValueError("Attention biases are not supported.")
        if cfg.get("hidden_act") != "silu":
            raise ValueError("Expected SiLU activation.")
        rope = cfg["rope_parameters"]
        if rope.get("rope_type") != "default":
            raise ValueError("Only default RoPE is supported.")
        c = cls(hidden=int(cfg["hidden_size"]), head_dim=int(cfg["head_dim"]),
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
                layer_types=list(cfg["layer_types"]))
        if c.value_heads % c.key_heads:
            raise ValueError("Value heads must be a multiple of key heads.")
        if c.heads % c.kv_heads:
            raise ValueError("Query heads must be a multiple of KV heads.")
        return c

    @property
    def key_width(self):
        return self.key_heads * self.key_dim

    @property
    def value_width(self):
        return self.value_heads * self.value_dim

    @property
    def qkv_width(self):
        return 2 * self.key_width + self.value_width


def read_safetensors(path, select=None, raw_bf16=False):
    """name -> float32 numpy array, row-major as stored (src/safetensors.jl:3-35).
    F32 / F16 widen exactly; BF16 widens as bits << 16 (:28-30), or with
    `raw_bf16` stays as its uint16 bits, to be copied to a device as they are
    and widened there (`device_f32`)."""
    out = {}
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        if not 0 < hlen <= size - 8:
            raise ValueError("Invalid safetensors header.")
        header = json.loads(f.read(hlen))
        base = 8 + hlen
        for name, spec in header.items():
            if name == "__metadata__" or (select is not None and not select(name)):
                continue
            start, stop = spec["data_offsets"]
            if not 0 <= start <= stop <= size - base:
                raise ValueError(f"Invalid offsets for tensor {name}.")
            dtype = {"F32": "<f4", "F16": "<f2", "BF16": "<u2"}.get(spec["dtype"])
            if dtype is None:
                raise ValueError(f"Native backend does not support tensor dtype {spec['dtype']}")
            shape = tuple(int(s) for s in spec["shape"])
            count = int(np.prod(shape)) if shape else 1
            if stop - start != count * np.dtype(dtype).itemsize:
                raise ValueError(f"Invalid size for tensor {name}.")
            f.seek(base + start)
            raw = np.frombuffer(f.read(stop - start), dtype)
            if spec["dtype"] == "BF16" and raw_bf16:
                arr = raw.copy()
            elif spec["dtype"] == "BF16":
                arr = (raw.astype(np.uint32) << 16).view(np.float32)
            else:
                arr = raw.astype(np.float32)
            out[name] = arr.reshape(shape)
    return out


def load_weights(directory, raw_bf16=False):
    """(Config, {canonical name: float32 array}) from a checkpoint directory:
    config.json + model.safetensors or the shards of
    model.safetensors.index.json, `language_model.` prefix canonicalised
    (src/backbone.jl:107-135).  `raw_bf16`: BF16 tensors stay uint16 bits
    (read_safetensors)."""
    with open(os.path.join(directory, "config.json")) as f:
        config = Config.from_json(json.load(f))
    single = os.path.join(directory, "model.safetensors")
    if os.path.isfile(single):
        files = [single]
    else:
        with open(os.path.join(directory, "model.safetensors.index.json")) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        for s in shards:
            if os.path.isabs(s) or ".." in s.split("/"):
                raise ValueError(f"unsafe shard path {s}")
        files = [os.path.join(directory, s) for s in shards]
    weights = {}
    for path in files:
        for name, value in read_safetensors(path, lambda n: "language_model." in n, raw_bf16).items():
            weights[name[name.find("language_model.") + len("language_model."):]] = value
    return config, weights


def random_weights(cfg, seed=0, std=0.02, device="cpu"):
    """Seeded random-init weights: linear N(0, std); zero-centred norm gammas
    N(0, std) (applied as 1+w); the DeltaNet output-norm gamma 1+N(0, std)
    (applied as w, src/backbone.jl:339); conv N(0, std); A_log U(-1, 0.5)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def n(*shape):
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)

    H, I = cfg.hidden, cfg.intermediate
    w = {"embed_tokens.weight": n(cfg.vocab, H), "norm.weight": n(H)}
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
        elif kind == "linear_attention":
            C = cfg.qkv_width
            w[p + "linear_attn.in_proj_qkv.weight"] = n(C, H)
            w[p + "linear_attn.in_proj_z.weight"] = n(cfg.value_width, H)
            w[p + "linear_attn.in_proj_a.weight"] = n(cfg.value_heads, H)
            w[p + "linear_attn.in_proj_b.weight"] = n(cfg.value_heads, H)
            w[p + "linear_attn.conv1d.weight"] = n(C, 1, cfg.conv_kernel)
            w[p + "linear_attn.A_log"] = torch.rand((cfg.value_heads,), generator=g, device=device,
                                                    dtype=torch.float32).mul_(1.5).sub_(1.0)
            w[p + "linear_attn.dt_bias"] = n(cfg.value_heads)
            w[p + "linear_attn.norm.weight"] = n(cfg.value_dim).add_(1.0)
            w[p + "linear_attn.out_proj.weight"] = n(H, cfg.value_width)
        else:
            raise ValueError(f"Unsupported layer type {kind}.")
    return w


def device_f32(x, device):
    """A Float32 tensor on `device` from a tensor or a numpy array.  uint16
    arrays are BF16 bits (read_safetensors(raw_bf16=True)): they are copied
    to the GPU as they are and widened there by qdc_bf16_to_f32, half the
    host -> device bytes of widening on the host."""
    if torch.is_tensor(x):
        return x.to(device=device, dtype=torch.float32).contiguous()
    if x.dtype == np.uint16:
        from . import ops
        bits = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(device)
        return ops.native_bf16_to_f32(bits)
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(device)


def pack_layers(cfg, weights, device):
    """Device weights per layer, projections packed so each block is one
    GEMM (the packing of ext/cuda_mlp.jl:9-47)."""
    layers = []
    take = lambda name: device_f32(weights[name], device)
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        layer = {
            "kind": "full" if kind == "full_attention" else "delta",
            "input_norm": take(p + "input_layernorm.weight"),
            "post_norm": take(p + "post_attention_layernorm.weight"),
            "gate_up": torch.cat([take(p + "mlp.gate_proj.weight"), take(p + "mlp.up_proj.weight")]),
            "down": take(p + "mlp.down_proj.weight"),
        }
        if kind == "full_attention":
            layer["qkv"] = torch.cat([take(p + "self_attn.q_proj.weight"),
                                      take(p + "self_attn.k_proj.weight"),
                                      take(p + "self_attn.v_proj.weight")])
            layer["out"] = take(p + "self_attn.o_proj.weight")
            layer["q_norm"] = take(p + "self_attn.q_norm.weight")
            layer["k_norm"] = take(p + "self_attn.k_norm.weight")
        else:
            layer["proj"] = torch.cat([take(p + "linear_attn.in_proj_qkv.weight"),
                                       take(p + "linear_attn.in_proj_z.weight"),
                                       take(p + "linear_attn.in_proj_a.weight"),
                                       take(p + "linear_attn.in_proj_b.weight")])
            conv = take(p + "linear_attn.conv1d.weight")
            layer["conv"] = conv.reshape(conv.shape[0], conv.shape[-1]).contiguous()
            # a_decay = -exp(A_log), precomputed once on the device (src/backbone.jl:160-162)
            layer["a_decay"] = -torch.exp(take(p + "linear_attn.A_log"))
            layer["dt_bias"] = take(p + "linear_attn.dt_bias")
            layer["norm"] = take(p + "linear_attn.norm.weight")
            layer["out"] = take(p + "linear_attn.out_proj.weight")
        layers.append(layer)
    return layers
