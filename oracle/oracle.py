"""numpy/ctypes front end of the CPU oracle (oracle/qdc_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline / reference arm, as the parity checker.  The product
(libqdc_b200.so and the qdc_b200 package) never imports this module.

Each wrapper restates one reference routine (cited in qdc_oracle.h) on
numpy arrays.  Layout: a Julia (width, tokens) matrix is a C-contiguous
numpy array of shape (tokens, width); strided views are passed with their
element strides, so q can be read straight out of a packed projection.
"""
import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libqdc_oracle.so")
_lock = threading.Lock()
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float

_SIGNATURES = {
    "qdo_set_threads": (None, [_int]),
    "qdo_get_threads": (_int, []),
    "qdo_bf16_encode_array": (None, [_u16p, _f32p, _i64]),
    "qdo_bf16_decode_array": (None, [_f32p, _u16p, _i64]),
    "qdo_gather_f32": (_int, [_f32p, _f32p, _i32p, _i64, _i64, _i64]),
    "qdo_gather_bf16": (_int, [_u16p, _u16p, _i32p, _i64, _i64, _i64]),
    "qdo_rms": (None, [_f32p, _f32p, _f32p, _flt, _int, _i64, _i64, _i64, _i64]),
    "qdo_residual_rms": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _flt, _int,
                                _i64, _i64, _i64, _i64, _i64, _i64]),
    "qdo_residual_rms_bf16": (None, [_u16p, _u16p, _u16p, _u16p, _f32p, _flt, _int,
                                     _i64, _i64, _i64, _i64, _i64, _i64]),
    "qdo_gather_rms_f32": (_int, [_f32p, _f32p, _f32p, _i32p, _f32p, _f32p, _flt,
                                  _int, _i64, _i64, _i64]),
    "qdo_gather_rms_bf16": (_int, [_u16p, _u16p, _u16p, _i32p, _u16p, _f32p, _flt,
                                   _int, _i64, _i64, _i64]),
    "qdo_rope_table": (None, [_flt, _int, _i64, _f32p, _f32p]),
    "qdo_qk_norm_rope": (None, [_f32p, _f32p, _i64, _int, _int, _i64, _i64, _f32p,
                                _flt, _int, _f32p, _f32p, _i64, _i64]),
    "qdo_gated_rms": (None, [_f32p, _f32p, _f32p, _i64, _int, _int, _i64, _i64,
                             _i64, _i64, _f32p, _flt]),
    "qdo_swiglu": (None, [_f32p, _u16p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
    "qdo_attn_gate": (None, [_f32p, _f32p, _f32p, _i64, _i64, _int, _int, _i64, _i64, _i64, _i64,
                             _i64, _i64]),
    "qdo_delta_gates": (None, [_f32p, _f32p, _f32p, _i64, _i64, _f32p, _f32p, _i64, _int]),
    "qdo_unit_lower_solve": (None, [_f32p, _f32p, _i64, _int, _i64, _i64, _i64, _i64, _i64]),
    "qdo_delta_conv_norm": (None, [_f32p, _f32p, _f32p, _f32p, _i64, _f32p, _i64, _i64, _int,
                                   _int, _int, _int, _flt]),
}


def build():
    """Compile oracle/_build/libqdc_oracle.so with oracle/Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                build()
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def set_threads(n):
    lib().qdo_set_threads(int(n))


def get_threads():
    return lib().qdo_get_threads()


def _p(a, kind=_f32p):
    return None if a is None else a.ctypes.data_as(kind)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _row_ld(a, itemsize):
    """Element stride between rows of a 2-D view with unit inner stride."""
    assert a.ndim == 2 and (a.shape[1] <= 1 or a.strides[1] == itemsize), a.strides
    return a.strides[0] // itemsize if a.shape[0] > 1 else a.shape[1]


# --- bf16, src/safetensors.jl:28-30, :38-42 --------------------------------

def bf16_encode(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().qdo_bf16_encode_array(_p(out, _u16p), _p(x), x.size)
    return out


def bf16_decode(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().qdo_bf16_decode_array(_p(out), _p(b, _u16p), b.size)
    return out


# --- gather, src/backbone.jl:55-64 -----------------------------------------

def gather(table, ids):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    vocab, hidden = table.shape
    if table.dtype == np.uint16:
        table = np.ascontiguousarray(table)
        out = np.empty((ids.size, hidden), np.uint16)
        rc = lib().qdo_gather_bf16(_p(out, _u16p), _p(table, _u16p), _p(ids, _i32p),
                                   ids.size, hidden, vocab)
    else:
        table = _f32(table)
        out = np.empty((ids.size, hidden), np.float32)
        rc = lib().qdo_gather_f32(_p(out), _p(table), _p(ids, _i32p), ids.size, hidden, vocab)
    if rc != 0:
        raise IndexError("Token ID is outside the vocabulary.")
    return out


# --- RMSNorm family ---------------------------------------------------------

def rms(x, weight, eps, centered=True):
    """src/backbone_cpu.jl:333-350 (centered) / src/backbone.jl:200-204."""
    x = _f32(x)
    rows, width = x.shape
    out = np.empty_like(x)
    lib().qdo_rms(_p(out), _p(x), _p(_f32(weight)), eps, int(centered), rows, width,
                  width, width)
    return out


def residual_rms(x, m, weight, eps, centered=True, store_residual=True):
    """src/backbone_cpu.jl:321-328: r = x + m; y = rms(r).  m may be None."""
    x = _f32(x)
    rows, width = x.shape
    m = None if m is None else _f32(m)
    r = np.empty_like(x) if store_residual else None
    y = np.empty_like(x)
    lib().qdo_residual_rms(_p(r), _p(y), _p(x), _p(m), _p(_f32(weight)), eps,
                           int(centered), rows, width, width, width, width, width)
    return r, y


def residual_rms_bf16(x, m, weight, eps, centered=True, store_residual=True):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    rows, width = x.shape
    m = None if m is None else np.ascontiguousarray(m, dtype=np.uint16)
    r = np.empty_like(x) if store_residual else None
    y = np.empty_like(x)
    lib().qdo_residual_rms_bf16(_p(r, _u16p), _p(y, _u16p), _p(x, _u16p), _p(m, _u16p),
                                _p(_f32(weight)), eps, int(centered), rows, width,
                                width, width, width, width)
    return r, y


def gather_rms(table, ids, m, weight, eps, centered=True, store_residual=True):
    """Gather (src/backbone.jl:55-64) + optional residual add + RMSNorm."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    vocab, hidden = table.shape
    n = ids.size
    if table.dtype == np.uint16:
        table = np.ascontiguousarray(table)
        m = None if m is None else np.ascontiguousarray(m, dtype=np.uint16)
        r = np.empty((n, hidden), np.uint16) if store_residual else None
        y = np.empty((n, hidden), np.uint16)
        rc = lib().qdo_gather_rms_bf16(_p(r, _u16p), _p(y, _u16p), _p(table, _u16p),
                                       _p(ids, _i32p), _p(m, _u16p), _p(_f32(weight)), eps,
                                       int(centered), n, hidden, vocab)
    else:
        table = _f32(table)
        m = None if m is None else _f32(m)
        r = np.empty((n, hidden), np.float32) if store_residual else None
        y = np.empty((n, hidden), np.float32)
        rc = lib().qdo_gather_rms_f32(_p(r), _p(y), _p(table), _p(ids, _i32p), _p(m),
                                      _p(_f32(weight)), eps, int(centered), n, hidden, vocab)
    if rc != 0:
        raise IndexError("Token ID is outside the vocabulary.")
    return r, y


# --- RoPE, src/backbone_cpu.jl:90-136 ---------------------------------------

def rope_table(theta, rotary, n):
    half = rotary // 2
    cos = np.empty((n, half), np.float32)
    sin = np.empty((n, half), np.float32)
    lib().qdo_rope_table(float(np.float32(theta)), int(rotary), int(n), _p(cos), _p(sin))
    return cos, sin


def qk_norm_rope(x, weight, eps, rotary, cos, sin, pos_offset=0, seq_len=None):
    """x: (tokens, heads, dim) float32 view, unit inner stride (may be a
    slice of a packed projection).  Returns dense (tokens, heads, dim)."""
    tokens, heads, dim = x.shape
    if x.size == 0:
        return np.empty((tokens, heads, dim), np.float32)
    assert x.dtype == np.float32 and x.ndim == 3 and x.strides[2] == 4
    cos = _f32(cos)
    sin = _f32(sin)
    half = rotary // 2
    if seq_len is None:
        seq_len = max(tokens, 1)
    if tokens:
        last = pos_offset + min(tokens, seq_len) - 1
        assert cos.shape[0] > last and cos.shape[1] == half
    out = np.empty((tokens, heads, dim), np.float32)
    in_tok = x.strides[0] // 4 if tokens > 1 else heads * dim
    in_head = x.strides[1] // 4 if heads > 1 else dim
    base = x.ctypes.data_as(_f32p)
    lib().qdo_qk_norm_rope(_p(out), base, tokens, heads, dim, in_tok, in_head,
                           _p(_f32(weight)), eps, int(rotary), _p(cos), _p(sin),
                           int(pos_offset), int(seq_len))
    return out


# --- gated RMSNorm, src/backbone_cpu.jl:750-755 -----------------------------

def gated_rms(o, z, weight, eps):
    """o, z: (rows, heads, dim) float32 views with unit inner stride and
    head stride dim (z may be a slice of the packed projection).  z is the
    raw projection; silu is applied here.  Returns (rows, heads*dim)."""
    assert o.shape == z.shape and o.ndim == 3
    rows, heads, dim = o.shape
    if o.size == 0:
        return np.empty((rows, heads * dim), np.float32)
    for a in (o, z):
        assert a.dtype == np.float32 and a.strides[2] == 4
        assert heads <= 1 or a.strides[1] == 4 * dim
    o_ld = o.strides[0] // 4 if rows > 1 else heads * dim
    z_ld = z.strides[0] // 4 if rows > 1 else heads * dim
    out = np.empty((rows, heads * dim), np.float32)
    lib().qdo_gated_rms(_p(out), o.ctypes.data_as(_f32p), z.ctypes.data_as(_f32p), rows,
                        heads, dim, o_ld, z_ld, 0, heads * dim, _p(_f32(weight)), eps)
    return out


# --- SwiGLU, src/backbone.jl:352-355 -----------------------------------------

def swiglu(g, u, want_f32=True, want_bf16=False):
    """g, u: (rows, width) float32 views with unit inner stride."""
    assert g.shape == u.shape and g.dtype == np.float32 and u.dtype == np.float32
    rows, width = g.shape
    if g.size == 0:
        return (np.empty((rows, width), np.float32) if want_f32 else None,
                np.empty((rows, width), np.uint16) if want_bf16 else None)
    out32 = np.empty((rows, width), np.float32) if want_f32 else None
    out16 = np.empty((rows, width), np.uint16) if want_bf16 else None
    lib().qdo_swiglu(_p(out32), _p(out16, _u16p), g.ctypes.data_as(_f32p),
                     u.ctypes.data_as(_f32p), rows, width, _row_ld(g, 4), _row_ld(u, 4),
                     width)
    return out32, out16


def delta_conv_norm(proj, conv_w, kh, kd, vh, vd, seq_len=None, eps=1e-6):
    """DeltaNet prologue (qdc_oracle.h): proj (tokens, >= channels) rows with
    unit inner stride, conv_w (channels, 4).  Returns q (tokens, kh, kd)
    normalised, k (tokens, kh, kd) normalised, v (tokens, vh, vd)."""
    assert proj.dtype == np.float32 and proj.ndim == 2
    tokens = proj.shape[0]
    C = 2 * kh * kd + vh * vd
    w = _f32(conv_w).reshape(C, 4)
    q = np.empty((tokens, kh, kd), np.float32)
    k = np.empty((tokens, kh, kd), np.float32)
    v = np.empty((tokens, vh, vd), np.float32)
    if tokens:
        lib().qdo_delta_conv_norm(_p(q), _p(k), _p(v), proj.ctypes.data_as(_f32p), _row_ld(proj, 4),
                                  _p(w), tokens, int(seq_len or tokens), kh, kd, vh, vd, eps)
    return q, k, v


def attn_gate(values, gate):
    """values (batch, heads, seq, dim) float32 view (unit inner stride), gate
    (batch*seq, heads, dim) view.  Returns out (batch*seq, heads*dim):
    values * sigmoid(gate), src/backbone.jl:258-259."""
    B, H, S, D = values.shape
    assert values.dtype == np.float32 and values.strides[3] == 4
    assert gate.shape == (B * S, H, D) and gate.dtype == np.float32 and gate.strides[2] == 4
    out = np.empty((B * S, H * D), np.float32)
    if out.size:
        st = [x // 4 for x in values.strides]
        lib().qdo_attn_gate(_p(out), values.ctypes.data_as(_f32p), gate.ctypes.data_as(_f32p), B, S,
                            H, D, st[0], st[1], st[2], gate.strides[0] // 4, gate.strides[1] // 4,
                            H * D)
    return out


def delta_gates(proj, start, heads, a_decay, dt_bias):
    """proj (tokens, >= start + 2 heads) float32 with unit inner stride.
    Returns (beta, decay), each (tokens, heads): sigmoid(b) and
    a_decay * softplus(a + dt_bias), src/backbone.jl:292-297."""
    assert proj.dtype == np.float32 and proj.ndim == 2
    assert proj.size == 0 or proj.strides[1] == 4
    assert start >= 0 and start + 2 * heads <= proj.shape[1]
    tokens = proj.shape[0] if proj.size else 0
    a_decay, dt_bias = _f32(a_decay).reshape(-1), _f32(dt_bias).reshape(-1)
    assert a_decay.size == heads and dt_bias.size == heads
    beta = np.empty((tokens, heads), np.float32)
    decay = np.empty((tokens, heads), np.float32)
    if tokens:
        lib().qdo_delta_gates(_p(beta), _p(decay), proj.ctypes.data_as(_f32p), proj.strides[0] // 4,
                              start, _p(a_decay), _p(dt_bias), tokens, heads)
    return beta, decay


def unit_lower_solve(system, rhs):
    """delta_solve (src/backbone.jl:279): UnitLowerTriangular(system) \\ rhs for
    a batch: system (batch, n, n), rhs (batch, n, width).  Returns the
    solution (batch, n, width) float32."""
    L = _f32(system)
    x = np.array(rhs, dtype=np.float32, order="C", copy=True)
    batch, n, width = x.shape
    assert L.shape == (batch, n, n)
    if x.size:
        lib().qdo_unit_lower_solve(_p(x), _p(L), batch, n, width, n, n * n, width, n * width)
    return x


def silu(x):
    """src/backbone.jl:196-197 elementwise, as SwiGLU with up = 1."""
    x = _f32(x)
    flat = x.reshape(1, -1) if x.size else x.reshape(0, 1)
    out, _ = swiglu(flat, np.ones_like(flat))
    return out.reshape(x.shape)
