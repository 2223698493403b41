"""ctypes binding of libqdc_b200.so (the C ABI in include/qdc_b200.h).

This is the Python twin of the `ccall` layer of the Julia extension
(qwendecisioncore.jl_b200/julia/QwenDecisionCoreB200Ext.jl): plain pointers, sizes and a
cudaStream_t, status codes turned into the reference's exception kinds
(ArgumentError / DimensionMismatch, src/backbone.jl:413-422).

There is no fallback: if the library is missing or fails to load, every
entry point raises.
"""
import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_PKG)
LIB_PATH = os.environ.get("QDC_B200_LIB", os.path.join(_ROOT, "_build", "libqdc_b200.so"))
HEADER_PATH = os.path.join(os.path.dirname(_ROOT), "include", "qdc_b200.h")

QDC_OK, QDC_EINVAL, QDC_EBOUNDS, QDC_ECUDA, QDC_ENOMEM, QDC_EDEVICE = range(6)
QDC_F32, QDC_BF16 = 0, 1
QDC_OPT_PDL = 1


class QdcError(RuntimeError):
    """A libqdc_b200 call failed; `status` is the qdc_status code."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class ArgumentError(QdcError, ValueError):
    """Bad arguments or out-of-vocabulary ids (Julia's ArgumentError)."""


class DimensionMismatch(QdcError, ValueError):
    """Shapes that do not fit together (Julia's DimensionMismatch)."""


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float
_sz = ctypes.c_size_t
_szp = ctypes.POINTER(ctypes.c_size_t)

# name -> argument types (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "qdc_abi_version": [],
    "qdc_status_string": [_int],
    "qdc_init": [_int, ctypes.POINTER(_vp)],
    "qdc_destroy": [_vp],
    "qdc_last_error": [_vp],
    "qdc_set_option": [_vp, _int, _int],
    "qdc_sync": [_vp, _vp],
    "qdc_ws_reserve": [_vp, _sz],
    "qdc_ws_alloc": [_vp, _sz, _sz, ctypes.POINTER(_vp)],
    "qdc_ws_mark": [_vp, _szp],
    "qdc_ws_release": [_vp, _sz],
    "qdc_ws_reset": [_vp],
    "qdc_ws_stats": [_vp, _szp, _szp, _szp],
    "qdc_rope_table": [_flt, _int, _i64, _vp, _vp],
    "qdc_gather": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp],
    "qdc_gather_rms": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _flt, _int, _i64, _i64, _i64, _int, _vp],
    "qdc_gather_rms_device_ids": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _flt, _int, _i64, _i64, _i64,
                                  _int, _vp],
    "qdc_gather_rms_noalloc": [_vp, _vp, _vp, _vp, _vp, _vp, _flt, _int, _i64, _i64, _i64, _int, _vp],
    "qdc_residual_rms": [_vp, _vp, _vp, _vp, _vp, _vp, _flt, _int, _i64, _i64, _i64, _i64, _i64,
                         _i64, _int, _vp],
    "qdc_qk_norm_rope": [_vp, _vp, _vp, _i64, _int, _int, _i64, _i64, _vp, _flt, _int, _vp, _vp,
                         _i64, _i64, _i64, _vp],
    "qdc_qk_norm_rope_strided": [_vp, _vp, _vp, _i64, _int, _int, _i64, _i64, _i64, _i64, _vp, _flt, _int,
                                 _vp, _vp, _i64, _i64, _i64, _vp],
    "qdc_q_k_norm_rope": [_vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64, _i64, _i64,
                          _vp, _vp, _flt, _int, _vp, _vp, _i64, _i64, _i64, _vp],
    "qdc_gated_rms": [_vp, _vp, _vp, _vp, _i64, _int, _int, _i64, _i64, _i64, _i64, _vp, _flt, _vp],
    "qdc_attn_gate": [_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _i64, _i64, _i64, _i64, _i64, _i64,
                      _vp],
    "qdc_bf16_to_f32": [_vp, _vp, _vp, _i64, _vp],
    "qdc_f32_to_bf16": [_vp, _vp, _vp, _i64, _vp],
    "qdc_delta_gates": [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _int, _vp],
    "qdc_delta_conv_norm": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _int, _int, _int, _int,
                            _flt, _vp],
    "qdc_delta_conv_norm_strided": [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _int, _int, _int,
                                    _int, _flt, _vp],
    "qdc_swiglu": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp],
    "qdc_unit_lower_solve": [_vp, _vp, _vp, _i64, _int, _i64, _i64, _i64, _i64, _i64, _vp],
}
_RESTYPES = {"qdc_status_string": ctypes.c_char_p, "qdc_last_error": ctypes.c_char_p}

_lock = threading.Lock()
_lib = None


def load(path=None):
    """Load (once) and return the ctypes handle; raises if it cannot."""
    global _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise OSError(f"libqdc_b200.so not found at {p}; run "
                              "`python qwendecisioncore.jl_b200/build.py` (or __graft_entry__.build())")
            handle = ctypes.CDLL(p)
            for name, args in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = handle
        return _lib


def declared_symbols(header=HEADER_PATH):
    """Names of the functions declared in include/qdc_b200.h."""
    import re
    with open(header) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*QDC_API\s+(?:int|const char \*)\s*(qdc_\w+)\s*\(", text, re.M)))


def check(status, ctx=None, exc=None):
    """Raise for a non-zero status with the library's error text."""
    if status == QDC_OK:
        return
    lib = load()
    msg = lib.qdc_last_error(ctx)
    msg = msg.decode() if msg else lib.qdc_status_string(status).decode()
    if exc is None:
        exc = ArgumentError if status in (QDC_EINVAL, QDC_EBOUNDS) else QdcError
    raise exc(status, msg)
