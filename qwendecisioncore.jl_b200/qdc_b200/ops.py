"""Tensor-level front end of libqdc_b200: the reference's per-layer hooks.

Each function mirrors one hook of the reference's forward core (name,
argument meaning and error behaviour), with torch CUDA tensors standing in
for CuArrays and the work done by the library's sm_100a kernels:

  native_gather        src/backbone.jl:55-64, ext/cuda_workspace.jl:330-344
  native_rms           src/backbone.jl:200-204, ext/cuda_workspace.jl:156-170
  native_residual_rms  src/backbone.jl:347-350, ext/cuda_workspace.jl:196-209
  native_residual_add_rms  native_residual_add! (src/backbone.jl:358-361)
                       fused with the next native_rms
  native_qk_norm_rope  native_rms + native_rope of full_attention,
                       src/backbone.jl:206-235 (CPU form src/backbone_cpu.jl:113-136)
  native_q_k_norm_rope the same for the query and key heads in one launch
  native_gated_rms     src/backbone.jl:339-341, ext/cuda_delta.jl:99-116
  native_attn_gate     values .* sigmoid(gate), src/backbone.jl:258-259,
                       ext/cuda_attention.jl:92-108
  native_delta_conv_norm  conv + SiLU + q/k L2 norms of delta_attention,
                       src/backbone.jl:287-314, ext/cuda_delta.jl:8-40,122-146
  native_delta_gates   beta / decay of delta_attention, src/backbone.jl:292-297,
                       ext/cuda_delta.jl:168-181
  native_mlp_gate      src/backbone.jl:352-355, ext/cuda_mlp.jl:49-61
  native_delta_solve   delta_solve (UnitLowerTriangular(system) \\ rhs) of the
                       chunked gated delta rule, src/backbone.jl:279,
                       ext/QwenDecisionCoreCUDAExt.jl:22-24
  native_bf16_to_f32   BF16 decode (bits << 16), src/safetensors.jl:28-30
  native_f32_to_bf16   BF16 encode (round to nearest even), src/safetensors.jl:38-42
  rope_table           src/backbone_cpu.jl:90-105

Layout: a Julia (width, tokens) matrix is a (tokens, width) row-major
tensor here.  Validation mirrors the reference: shape errors raise
DimensionMismatch, bad ids / values raise ArgumentError, before any launch.
Tensors must live on a CUDA device; there is no CPU path.
"""
import ctypes
import threading

import torch

from . import _lib
from ._lib import ArgumentError, DimensionMismatch, QDC_BF16, QDC_F32, check

_ctx_lock = threading.Lock()
_contexts = {}


class Context:
    """A libqdc_b200 context on one device: workspace arena + error flag.

    Mirrors the reference's per-model ForwardWorkspace
    (ext/cuda_workspace.jl:4-46): one forward at a time per context."""

    def __init__(self, device):
        self.lib = _lib.load()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ArgumentError(_lib.QDC_EINVAL, f"libqdc_b200 needs a CUDA device, got {self.device}")
        handle = ctypes.c_void_p()
        check(self.lib.qdc_init(self.device.index or 0, ctypes.byref(handle)))
        self.handle = handle
        self.lock = threading.RLock()
        self._pdl = True

    @property
    def pdl(self):
        """Programmatic dependent launch of this context's kernels (on by
        default; QDC_OPT_PDL of include/qdc_b200.h)."""
        return self._pdl

    @pdl.setter
    def pdl(self, on):
        check(self.lib.qdc_set_option(self.handle, _lib.QDC_OPT_PDL, int(bool(on))), self.handle)
        self._pdl = bool(on)

    def close(self):
        if self.handle:
            self.lib.qdc_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self, stream=None):
        """Synchronize and report a device-side out-of-vocabulary flag."""
        check(self.lib.qdc_sync(self.handle, _stream(self.device, stream)), self.handle)

    # -- workspace arena (replaces ext/cuda_workspace.jl:71-87) -------------
    def ws_reserve(self, nbytes):
        check(self.lib.qdc_ws_reserve(self.handle, int(nbytes)), self.handle)

    def ws_alloc(self, nbytes, align=256):
        p = ctypes.c_void_p()
        check(self.lib.qdc_ws_alloc(self.handle, int(nbytes), int(align), ctypes.byref(p)),
              self.handle)
        return p.value

    def ws_mark(self):
        m = ctypes.c_size_t()
        check(self.lib.qdc_ws_mark(self.handle, ctypes.byref(m)), self.handle)
        return m.value

    def ws_release(self, mark):
        check(self.lib.qdc_ws_release(self.handle, int(mark)), self.handle)

    def ws_reset(self):
        check(self.lib.qdc_ws_reset(self.handle), self.handle)

    def ws_stats(self):
        used, cap, high = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        check(self.lib.qdc_ws_stats(self.handle, ctypes.byref(used), ctypes.byref(cap),
                                    ctypes.byref(high)), self.handle)
        return used.value, cap.value, high.value

    def ws_tensor(self, shape, dtype=torch.float32):
        """A tensor view of freshly carved arena memory (no torch allocation)."""
        numel = 1
        for s in shape:
            numel *= int(s)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        ptr = self.ws_alloc(max(nbytes, 1))
        return self.wrap(ptr, shape, dtype)

    def wrap(self, ptr, shape, dtype=torch.float32):
        """A tensor view of `shape` over device memory at `ptr` (not owned)."""
        return _wrap_device_pointer(ptr, tuple(int(s) for s in shape), dtype, self.device)


def context(device=None):
    """The shared context of `device` (current CUDA device by default)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    with _ctx_lock:
        ctx = _contexts.get(dev.index)
        if ctx is None:
            ctx = _contexts[dev.index] = Context(dev)
        return ctx


_TORCH_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<u2", torch.int32: "<i4",
                  torch.uint8: "|u1", torch.int64: "<i8", torch.bool: "|b1"}


class _CudaArray:
    def __init__(self, ptr, shape, dtype):
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": _TORCH_TYPESTR[dtype], "data": (ptr, False), "version": 3,
            "strides": None}


def _wrap_device_pointer(ptr, shape, dtype, device):
    with torch.cuda.device(device):
        t = torch.as_tensor(_CudaArray(ptr, shape, dtype), device=device)
    if dtype == torch.bfloat16:
        t = t.view(torch.bfloat16)
    return t


def _stream(device, stream=None):
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


def _dtype_code(t):
    if t.dtype == torch.float32:
        return QDC_F32
    if t.dtype == torch.bfloat16:
        return QDC_BF16
    raise ArgumentError(_lib.QDC_EINVAL, f"unsupported storage dtype {t.dtype}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _cuda(*tensors):
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ArgumentError(_lib.QDC_EINVAL, "libqdc_b200 ops take CUDA tensors (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ArgumentError(_lib.QDC_EINVAL, "tensors live on different devices")
    return dev


def _rows(t, name):
    """(rows, width, ld) of a 2-D tensor with unit inner stride."""
    if t.dim() != 2:
        raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if t.numel() == 0:
        return t.shape[0], t.shape[1], max(t.shape[1], 1)
    if t.shape[1] > 1 and t.stride(1) != 1:
        raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} needs a unit inner stride")
    ld = t.stride(0) if t.shape[0] > 1 else t.shape[1]
    return t.shape[0], t.shape[1], ld


def _gamma(weight, width, dev):
    if weight.dim() != 1 or weight.shape[0] != width:
        raise DimensionMismatch(_lib.QDC_EINVAL, "RMS weight width differs.")
    if weight.dtype != torch.float32 or weight.device != dev:
        raise ArgumentError(_lib.QDC_EINVAL, "gamma must be a Float32 tensor on the same device")
    return weight.contiguous()


# --------------------------------------------------------------------- ops

def native_gather_rms(embedding, ids, weight=None, eps=1e-6, *, add=None, centered=True,
                      store_x=True, ctx=None, out_x=None, out_y=None, stream=None):
    """r_t = E[ids_t] (+ add_t), y_t = rms(r_t): the gather of
    src/backbone.jl:55-64 fused with the first layer's input norm.

    `ids` may be a host sequence / CPU tensor (validated and staged, as the
    reference does, ext/cuda_workspace.jl:330-334) or an int32 CUDA tensor
    (device-checked; out-of-range rows poisoned and reported by ctx.sync()).
    Returns (x or None, y or None)."""
    dev = _cuda(embedding, weight, add, out_x, out_y)
    vocab, hidden, ld_e = _rows(embedding, "embedding")
    if ld_e != hidden:
        raise DimensionMismatch(_lib.QDC_EINVAL, "embedding must be contiguous")
    ctx = ctx or context(dev)
    device_ids = torch.is_tensor(ids) and ids.is_cuda
    if device_ids:
        if ids.dtype != torch.int32 or ids.dim() != 1:
            raise ArgumentError(_lib.QDC_EINVAL, "device ids must be a 1-D int32 tensor")
        ids = ids.contiguous()
        n = ids.shape[0]
    else:
        host = torch.as_tensor(ids, dtype=torch.int64).reshape(-1)
        n = host.shape[0]
        if n and (int(host.min()) < 0 or int(host.max()) >= vocab):
            raise ArgumentError(_lib.QDC_EBOUNDS, "Token ID is outside the vocabulary.")
        host32 = host.to(torch.int32).contiguous()
    if weight is not None:
        weight = _gamma(weight, hidden, dev)
    if add is not None:
        if tuple(add.shape) != (n, hidden) or add.dtype != embedding.dtype:
            raise DimensionMismatch(_lib.QDC_EINVAL, "residual shape/dtype differs from the gather")
        add = add.contiguous()
    if store_x and out_x is None:
        out_x = torch.empty((n, hidden), dtype=embedding.dtype, device=dev)
    if weight is not None and out_y is None:
        out_y = torch.empty((n, hidden), dtype=embedding.dtype, device=dev)
    for t in (out_x, out_y):
        if t is not None and (tuple(t.shape) != (n, hidden) or not t.is_contiguous()
                              or t.dtype != embedding.dtype):
            raise DimensionMismatch(_lib.QDC_EINVAL, "output shape/dtype differs")
    dt = _dtype_code(embedding)
    with ctx.lock:
        if device_ids:
            st = ctx.lib.qdc_gather_rms_device_ids(
                ctx.handle, _ptr(out_x), _ptr(out_y), _ptr(embedding), _ptr(ids), _ptr(add),
                _ptr(weight), float(eps), int(bool(centered)), n, hidden, vocab, dt,
                _stream(dev, stream))
        else:
            st = ctx.lib.qdc_gather_rms(
                ctx.handle, _ptr(out_x), _ptr(out_y), _ptr(embedding),
                host32.data_ptr() if n else None, _ptr(add), _ptr(weight), float(eps),
                int(bool(centered)), n, hidden, vocab, dt, _stream(dev, stream))
        check(st, ctx.handle)
    return out_x, out_y


def native_gather(embedding, ids, **kw):
    """hidden[t, :] = embedding[ids[t], :] bit for bit, src/backbone.jl:55-64."""
    x, _ = native_gather_rms(embedding, ids, None, store_x=True, **kw)
    return x


def native_residual_rms(x, mixed, weight, eps, *, centered=True, store_residual=True, out_r=None,
                        out_y=None, inplace=False, ctx=None, stream=None):
    """residual = x + mixed; normalized = rms(residual); returns
    (residual or None, normalized).  `mixed` None gives native_rms of x.
    `inplace=True` writes the residual back into x (the reference reuses the
    layer-owned residual the same way, src/backbone.jl:377-381)."""
    dev = _cuda(x, mixed, weight, out_r, out_y)
    rows, width, ld_x = _rows(x, "x")
    ld_m = 0
    if mixed is not None:
        if tuple(mixed.shape) != (rows, width) or mixed.dtype != x.dtype:
            raise DimensionMismatch(_lib.QDC_EINVAL, "residual shapes differ")
        _, _, ld_m = _rows(mixed, "mixed")
    weight = _gamma(weight, width, dev)
    if inplace:
        out_r = x
    elif store_residual and out_r is None:
        out_r = torch.empty((rows, width), dtype=x.dtype, device=dev)
    if not store_residual and not inplace:
        out_r = None
    if out_y is None:
        out_y = torch.empty((rows, width), dtype=x.dtype, device=dev)
    ld_r = _rows(out_r, "out_r")[2] if out_r is not None else width
    ld_y = _rows(out_y, "out_y")[2]
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_residual_rms(ctx.handle, _ptr(out_r), _ptr(out_y), _ptr(x), _ptr(mixed),
                                       _ptr(weight), float(eps), int(bool(centered)), rows, width,
                                       ld_x, ld_m, ld_r, ld_y, _dtype_code(x), _stream(dev, stream)),
              ctx.handle)
    return out_r, out_y


def native_rms(x, weight, eps, *, centered=True, out=None, ctx=None, stream=None):
    """y = x * inv(sqrt(sum(x^2)/width + eps)) * (1 + w) (or * w uncentered),
    per row: src/backbone.jl:200-204."""
    _, y = native_residual_rms(x, None, weight, eps, centered=centered, store_residual=False,
                               out_y=out, ctx=ctx, stream=stream)
    return y


def native_residual_add_rms(residual, mlp_out, next_weight, eps, *, out_y=None, store_residual=True,
                            ctx=None, stream=None):
    """native_residual_add! (src/backbone.jl:358-361) fused with the next
    layer's input norm (or the final norm, :410): residual += mlp_out in
    place, returns (residual, rms(residual))."""
    return native_residual_rms(residual, mlp_out, next_weight, eps, inplace=store_residual,
                               store_residual=store_residual, out_y=out_y, ctx=ctx, stream=stream)


def rope_table(theta, rotary, n, device=None):
    """(cos, sin), each (n, rotary/2) Float32, built on the host exactly as
    src/backbone_cpu.jl:90-105 and copied to `device` (None: CPU tensors)."""
    lib = _lib.load()
    half = int(rotary) // 2
    cos = torch.empty((int(n), half), dtype=torch.float32)
    sin = torch.empty((int(n), half), dtype=torch.float32)
    check(lib.qdc_rope_table(float(theta), int(rotary), int(n),
                             ctypes.c_void_p(cos.data_ptr()) if cos.numel() else None,
                             ctypes.c_void_p(sin.data_ptr()) if sin.numel() else None))
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin


def native_qk_norm_rope(x, weight, eps, rotary, cos, sin, *, pos_offset=0, seq_len=None, out=None,
                        ctx=None, stream=None):
    """Per-head RMSNorm (1+w) then rotate-half RoPE on the first `rotary`
    dims.  x: (tokens, heads, dim) view with unit inner stride -- q may be
    qgate[:, :, :dim] of the packed (tokens, heads, 2*dim) projection.
    Position of token t: pos_offset + t % seq_len (seq_len None: t).
    Returns dense (tokens, heads, dim)."""
    dev = _cuda(x, weight, cos, sin, out)
    if x.dim() != 3 or (x.numel() and x.shape[2] > 1 and x.stride(2) != 1):
        raise DimensionMismatch(_lib.QDC_EINVAL, "x must be (tokens, heads, dim) with unit inner stride")
    if x.dtype != torch.float32:
        raise ArgumentError(_lib.QDC_EINVAL, "q/k norm takes Float32 projections")
    tokens, heads, dim = x.shape
    weight = _gamma(weight, dim, dev)
    if rotary % 2 or rotary > dim or rotary < 0:
        raise ArgumentError(_lib.QDC_EINVAL, "rotary dims must be even and <= head_dim")
    rows = 0
    if rotary > 0:
        if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != rotary // 2:
            raise DimensionMismatch(_lib.QDC_EINVAL, "RoPE table shape differs")
        cos, sin = cos.contiguous(), sin.contiguous()
        rows = cos.shape[0]
    if out is None:
        out = torch.empty((tokens, heads, dim), dtype=torch.float32, device=dev)
    elif tuple(out.shape) != (tokens, heads, dim) or (out.numel() and dim > 1 and out.stride(2) != 1):
        raise DimensionMismatch(_lib.QDC_EINVAL, "output must be (tokens, heads, dim) with unit inner stride")
    in_tok = x.stride(0) if tokens > 1 else heads * dim
    in_head = x.stride(1) if heads > 1 else dim
    # any output strides (e.g. a head-major (heads, tokens, dim) buffer seen
    # as (tokens, heads, dim)); dense outputs take the same kernel
    out_tok = out.stride(0) if tokens > 1 else heads * dim
    out_head = out.stride(1) if heads > 1 else dim
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_qk_norm_rope_strided(
            ctx.handle, _ptr(out), _ptr(x), tokens, heads, dim, in_tok, in_head, out_tok, out_head,
            _ptr(weight), float(eps), int(rotary), _ptr(cos) if rotary else None,
            _ptr(sin) if rotary else None, rows, int(pos_offset), int(seq_len or 0), _stream(dev, stream)),
            ctx.handle)
    return out


def native_q_k_norm_rope(q_in, k_in, q_weight, k_weight, eps, rotary, cos, sin, *, pos_offset=0,
                        seq_len=None, q_out=None, k_out=None, ctx=None, stream=None):
    """The query and key halves of native_qk_norm_rope in ONE launch:
    q_in (tokens, q_heads, dim), k_in (tokens, k_heads, dim) views (e.g. both
    slices of the packed [q;gate | k | v] projection).  Returns dense
    (q, k)."""
    dev = _cuda(q_in, k_in, q_weight, k_weight, cos, sin, q_out, k_out)
    for x, name in ((q_in, "q"), (k_in, "k")):
        if x.dim() != 3 or (x.numel() and x.shape[2] > 1 and x.stride(2) != 1):
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} must be (tokens, heads, dim) with unit "
                                                     "inner stride")
        if x.dtype != torch.float32:
            raise ArgumentError(_lib.QDC_EINVAL, "q/k norm takes Float32 projections")
    tokens, qh, dim = q_in.shape
    if k_in.shape[0] != tokens or k_in.shape[2] != dim:
        raise DimensionMismatch(_lib.QDC_EINVAL, "q and k shapes differ")
    kh = k_in.shape[1]
    q_weight, k_weight = _gamma(q_weight, dim, dev), _gamma(k_weight, dim, dev)
    if rotary % 2 or rotary > dim or rotary < 0:
        raise ArgumentError(_lib.QDC_EINVAL, "rotary dims must be even and <= head_dim")
    rows = 0
    if rotary > 0:
        if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != rotary // 2:
            raise DimensionMismatch(_lib.QDC_EINVAL, "RoPE table shape differs")
        cos, sin = cos.contiguous(), sin.contiguous()
        rows = cos.shape[0]
    if q_out is None:
        q_out = torch.empty((tokens, qh, dim), dtype=torch.float32, device=dev)
    if k_out is None:
        k_out = torch.empty((tokens, kh, dim), dtype=torch.float32, device=dev)
    for t, shape in ((q_out, (tokens, qh, dim)), (k_out, (tokens, kh, dim))):
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise DimensionMismatch(_lib.QDC_EINVAL, "output shape differs")
    strides = []
    for x, heads in ((q_in, qh), (k_in, kh)):
        strides.append(x.stride(0) if tokens > 1 else heads * dim)
        strides.append(x.stride(1) if heads > 1 else dim)
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_q_k_norm_rope(
            ctx.handle, _ptr(q_out), _ptr(k_out), _ptr(q_in), _ptr(k_in), tokens, qh, kh, dim,
            strides[0], strides[1], strides[2], strides[3], _ptr(q_weight), _ptr(k_weight),
            float(eps), int(rotary), _ptr(cos) if rotary else None, _ptr(sin) if rotary else None,
            rows, int(pos_offset), int(seq_len or 0), _stream(dev, stream)), ctx.handle)
    return q_out, k_out


def native_gated_rms(o, z, weight, eps, *, out=None, ctx=None, stream=None):
    """normalized(o) * w * silu(z) per (row, head), uncentered w:
    src/backbone.jl:339-341.  o, z: (rows, heads, dim) views (unit inner
    stride, head stride dim; z may be a slice of the packed projection).
    Returns (rows, heads*dim)."""
    dev = _cuda(o, z, weight, out)
    if o.dim() != 3 or tuple(z.shape) != tuple(o.shape):
        raise DimensionMismatch(_lib.QDC_EINVAL, "o and z must both be (rows, heads, dim)")
    rows, heads, dim = o.shape
    for t, name in ((o, "o"), (z, "z")):
        if t.dtype != torch.float32:
            raise ArgumentError(_lib.QDC_EINVAL, f"{name} must be Float32")
        if t.numel() and ((dim > 1 and t.stride(2) != 1) or (heads > 1 and t.stride(1) != dim)):
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} needs contiguous heads within a row")
    weight = _gamma(weight, dim, dev)
    if out is None:
        out = torch.empty((rows, heads * dim), dtype=torch.float32, device=dev)
    _, _, ld_out = _rows(out, "out")
    o_ld = o.stride(0) if rows > 1 else heads * dim
    z_ld = z.stride(0) if rows > 1 else heads * dim
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_gated_rms(ctx.handle, _ptr(out), _ptr(o), _ptr(z), rows, heads, dim, o_ld,
                                    z_ld, 0, ld_out, _ptr(weight), float(eps), _stream(dev, stream)),
              ctx.handle)
    return out


def native_attn_gate(values, gate, *, out=None, ctx=None, stream=None):
    """values * sigmoid(gate) (src/backbone.jl:258-259): values is the
    attention output (batch, heads, seq, dim) in any strides with unit inner
    stride; gate (batch*seq, heads, dim) -- e.g. qgate[:, :, dim:] of the
    packed projection.  Returns (batch*seq, heads*dim)."""
    dev = _cuda(values, gate, out)
    if values.dim() != 4 or gate.dim() != 3:
        raise DimensionMismatch(_lib.QDC_EINVAL, "values (B, H, S, D) and gate (B*S, H, D) expected")
    B, H, S, D = values.shape
    if tuple(gate.shape) != (B * S, H, D):
        raise DimensionMismatch(_lib.QDC_EINVAL, "gate shape differs from the attention output")
    for t, name in ((values, "values"), (gate, "gate")):
        if t.dtype != torch.float32:
            raise ArgumentError(_lib.QDC_EINVAL, f"{name} must be Float32")
        if t.numel() and D > 1 and t.stride(-1) != 1:
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} needs a unit inner stride")
    if out is None:
        out = torch.empty((B * S, H * D), dtype=torch.float32, device=dev)
    _, _, out_t = _rows(out, "out")
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_attn_gate(ctx.handle, _ptr(out), _ptr(values), _ptr(gate), B, S, H, D,
                                    values.stride(0), values.stride(1), values.stride(2),
                                    gate.stride(0), gate.stride(1), out_t, _stream(dev, stream)),
              ctx.handle)
    return out


_BF16_BITS = (torch.bfloat16, torch.int16, torch.uint16)


def native_bf16_to_f32(bits, *, out=None, ctx=None, stream=None):
    """Float32 = bf16 bits << 16 (src/safetensors.jl:28-30), on the device:
    `bits` is a contiguous CUDA tensor of bfloat16 or of raw 16-bit words
    (int16 / uint16), e.g. a checkpoint's BF16 bytes copied as they are.
    Returns a Float32 tensor of the same shape."""
    dev = _cuda(bits, out)
    if bits.dtype not in _BF16_BITS or not bits.is_contiguous():
        raise ArgumentError(_lib.QDC_EINVAL, "bits must be a contiguous bfloat16 / int16 / uint16 tensor")
    if out is None:
        out = torch.empty(bits.shape, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != bits.numel():
        raise DimensionMismatch(_lib.QDC_EINVAL, "out must be a contiguous Float32 tensor of as many elements")
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_bf16_to_f32(ctx.handle, _ptr(out), _ptr(bits), bits.numel(), _stream(dev, stream)),
              ctx.handle)
    return out


def native_f32_to_bf16(x, *, out=None, ctx=None, stream=None):
    """bf16 storage of Float32 `x` by the reference's round-to-nearest-even
    integer add, no NaN special case (src/safetensors.jl:38-42).  Returns a
    bfloat16 tensor of the same shape (`out` may be bfloat16 / int16 / uint16)."""
    dev = _cuda(x, out)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ArgumentError(_lib.QDC_EINVAL, "x must be a contiguous Float32 tensor")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=dev)
    elif out.dtype not in _BF16_BITS or not out.is_contiguous() or out.numel() != x.numel():
        raise DimensionMismatch(_lib.QDC_EINVAL, "out must be a contiguous 16-bit tensor of as many elements")
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_f32_to_bf16(ctx.handle, _ptr(out), _ptr(x), x.numel(), _stream(dev, stream)),
              ctx.handle)
    return out


def native_delta_gates(proj, start, heads, a_decay, dt_bias, *, beta=None, decay=None, ctx=None,
                       stream=None):
    """beta = sigmoid(b), decay = a_decay * softplus(a + dt_bias) per (token,
    head) (src/backbone.jl:292-297), a = proj[:, start:start+heads] and b =
    proj[:, start+heads:start+2*heads] read in place.  Returns dense
    (tokens, heads) beta and decay."""
    dev = _cuda(proj, a_decay, dt_bias, beta, decay)
    if proj.dtype != torch.float32:
        raise ArgumentError(_lib.QDC_EINVAL, "proj must be Float32")
    tokens, width, ld = _rows(proj, "proj")
    if start < 0 or heads < 1 or start + 2 * heads > width:
        raise DimensionMismatch(_lib.QDC_EINVAL, "a and b columns fall outside proj")
    for t, name in ((a_decay, "a_decay"), (dt_bias, "dt_bias")):
        if t.dtype != torch.float32 or t.numel() != heads or (heads > 1 and t.stride(-1) != 1):
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} must be {heads} contiguous Float32 values")
    outs = []
    for t, name in ((beta, "beta"), (decay, "decay")):
        if t is None:
            t = torch.empty((tokens, heads), dtype=torch.float32, device=dev)
        elif t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != tokens * heads:
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} must be a dense ({tokens}, {heads}) Float32")
        outs.append(t)
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_delta_gates(ctx.handle, _ptr(outs[0]), _ptr(outs[1]), _ptr(proj), ld, int(start),
                                      _ptr(a_decay), _ptr(dt_bias), tokens, int(heads),
                                      _stream(dev, stream)), ctx.handle)
    return outs[0], outs[1]


def native_delta_conv_norm(proj, conv_w, key_heads, key_dim, value_heads, value_dim, *, seq_len=None,
                           eps=1e-6, q_out=None, k_out=None, v_out=None, ctx=None, stream=None):
    """The Gated DeltaNet's row work after its projection GEMM, in one pass:
    causal 4-tap depthwise conv + SiLU over the [q | k | v] channels at the
    start of each row of `proj` (tokens, >= channels), then per-head L2
    normalisation of q (also / sqrt(key_dim)) and k
    (src/backbone.jl:287-314; CPU src/backbone_cpu.jl:787-807, :411-427).
    Sequences of `seq_len` tokens are packed back to back.  conv_w:
    (channels, 4) or the torch (channels, 1, 4).  Returns dense q, k
    (tokens, key_heads, key_dim) and v (tokens, value_heads, value_dim)."""
    dev = _cuda(proj, conv_w, q_out, k_out, v_out)
    tokens, width, ld = _rows(proj, "proj")
    C = 2 * key_heads * key_dim + value_heads * value_dim
    if width < C:
        raise DimensionMismatch(_lib.QDC_EINVAL, f"projection has {width} < {C} channels")
    if proj.dtype != torch.float32 or conv_w.dtype != torch.float32:
        raise ArgumentError(_lib.QDC_EINVAL, "DeltaNet prologue takes Float32 tensors")
    w = conv_w.reshape(conv_w.shape[0], conv_w.shape[-1]).contiguous()
    if tuple(w.shape) != (C, 4):
        raise DimensionMismatch(_lib.QDC_EINVAL, f"conv weight must be ({C}, 4), got {tuple(conv_w.shape)}")
    f = dict(dtype=torch.float32, device=dev)
    q_out = torch.empty((tokens, key_heads, key_dim), **f) if q_out is None else q_out
    k_out = torch.empty((tokens, key_heads, key_dim), **f) if k_out is None else k_out
    v_out = torch.empty((tokens, value_heads, value_dim), **f) if v_out is None else v_out
    for t, shape in ((q_out, (tokens, key_heads, key_dim)), (k_out, (tokens, key_heads, key_dim))):
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise DimensionMismatch(_lib.QDC_EINVAL, "output shape differs")
    # v may be a token-strided view (heads contiguous within a token), e.g.
    # the value rows of a wider buffer
    if tuple(v_out.shape) != (tokens, value_heads, value_dim) or (
            v_out.numel() and (v_out.stride(2) != 1 or (value_heads > 1 and v_out.stride(1) != value_dim))):
        raise DimensionMismatch(_lib.QDC_EINVAL, "v_out must be (tokens, value_heads, value_dim), heads contiguous")
    v_tok = v_out.stride(0) if tokens > 1 else value_heads * value_dim
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_delta_conv_norm_strided(ctx.handle, _ptr(q_out), _ptr(k_out), _ptr(v_out), v_tok,
                                                  _ptr(proj), ld, _ptr(w), tokens, int(seq_len or 0), key_heads,
                                                  key_dim, value_heads, value_dim, float(eps),
                                                  _stream(dev, stream)), ctx.handle)
    return q_out, k_out, v_out


def native_mlp_gate(gate, up, *, want_f32=True, want_bf16=False, out_f32=None, out_bf16=None,
                    ctx=None, stream=None):
    """silu(gate) * up (src/backbone.jl:352-355); gate/up (rows, width)
    views, e.g. the two halves of the packed (rows, 2*width) projection.
    Returns (Float32 or None, bf16 or None)."""
    dev = _cuda(gate, up, out_f32, out_bf16)
    if tuple(gate.shape) != tuple(up.shape):
        raise DimensionMismatch(_lib.QDC_EINVAL, "gate and up shapes differ")
    if gate.dtype != torch.float32 or up.dtype != torch.float32:
        raise ArgumentError(_lib.QDC_EINVAL, "SwiGLU takes Float32 projections")
    rows, width, ld_g = _rows(gate, "gate")
    _, _, ld_u = _rows(up, "up")
    if want_f32 and out_f32 is None:
        out_f32 = torch.empty((rows, width), dtype=torch.float32, device=dev)
    if want_bf16 and out_bf16 is None:
        out_bf16 = torch.empty((rows, width), dtype=torch.bfloat16, device=dev)
    if out_f32 is None and out_bf16 is None:
        raise ArgumentError(_lib.QDC_EINVAL, "no output requested")
    ld_out = width
    for t in (out_f32, out_bf16):
        if t is not None:
            if tuple(t.shape) != (rows, width) or not t.is_contiguous():
                raise DimensionMismatch(_lib.QDC_EINVAL, "output shape differs")
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_swiglu(ctx.handle, _ptr(out_f32), _ptr(out_bf16), _ptr(gate), _ptr(up),
                                 rows, width, ld_g, ld_u, ld_out, _stream(dev, stream)), ctx.handle)
    return out_f32, out_bf16


def native_delta_solve(system, x, *, ctx=None, stream=None):
    """x <- UnitLowerTriangular(system) \\ x in place for a batch (delta_solve,
    src/backbone.jl:279): system (batch, n, n) and x (batch, n, width)
    Float32 views with unit inner stride, n <= 64; the diagonal and upper
    triangle of system are not read.  Returns x."""
    dev = _cuda(system, x)
    if system.dim() != 3 or x.dim() != 3 or system.shape[0] != x.shape[0] \
            or system.shape[1] != system.shape[2] or x.shape[1] != system.shape[1]:
        raise DimensionMismatch(_lib.QDC_EINVAL, "system (batch, n, n) and x (batch, n, width) expected")
    if system.dtype != torch.float32 or x.dtype != torch.float32:
        raise ArgumentError(_lib.QDC_EINVAL, "delta_solve takes Float32 tensors")
    batch, n, width = x.shape
    if x.numel() == 0:
        return x
    for t, name in ((system, "system"), (x, "x")):
        if t.shape[2] > 1 and t.stride(2) != 1:
            raise DimensionMismatch(_lib.QDC_EINVAL, f"{name} needs a unit inner stride")
    ctx = ctx or context(dev)
    with ctx.lock:
        check(ctx.lib.qdc_unit_lower_solve(ctx.handle, _ptr(x), _ptr(system), batch, n, width,
                                           system.stride(1), system.stride(0), x.stride(1), x.stride(0),
                                           _stream(dev, stream)), ctx.handle)
    return x
