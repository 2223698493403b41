"""qdc_gather_rms_noalloc -- the gather + input norm for callers that may not
allocate device memory (hosts whose memory pool owns every device byte,
loops that cannot take cudaMalloc's device-wide synchronisation, fixed
memory budgets).  It needs no context and keeps its id staging in a fixed
array inside the library.

Called here through the C ABI (ctypes) and compared with the context-based
entry point, qdc_gather_rms, on consecutive calls (the second call must not
see anything of the first: the shared array keeps the last call's
contents), with the CPU oracle at every kernel shape it can take, and for
device memory: after the first call on a device, further calls leave the
device's free memory unchanged.  This file sorts last so a
stop-at-first-failure run has run everything else first; it also passes
alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _case(seed, n, hidden, vocab, with_add, dtype):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    table = torch.randn((vocab, hidden), generator=g, device="cuda").mul_(0.02).to(dtype)
    add = torch.randn((n, hidden), generator=g, device="cuda").to(dtype) if with_add else None
    gamma = torch.randn((hidden,), generator=g, device="cuda").mul_(0.02)
    ids = np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)
    return table, add, gamma, ids


def _code(dtype):
    import qdc_b200
    return qdc_b200.QDC_F32 if dtype == torch.float32 else qdc_b200.QDC_BF16


def _nan(n, hidden, dtype):
    return torch.full((n, hidden), float("nan"), device="cuda").to(dtype)


def _noalloc(lib, x, y, table, add, gamma, ids):
    n, hidden, vocab = ids.size, table.shape[1], table.shape[0]
    st = lib.qdc_gather_rms_noalloc(_vp(x), _vp(y), _vp(table), ids.ctypes.data_as(ctypes.c_void_p),
                                    _vp(add), _vp(gamma), 1e-6, 1, n, hidden, vocab, _code(table.dtype),
                                    _stream())
    assert st == 0, lib.qdc_last_error(None)


def _host(t):
    return t.float().cpu().numpy()


def _close(a, b, rtol):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return bool((np.abs(a - b) <= 1e-6 + rtol * np.abs(b)).all())


def test_noalloc_matches_context_entry_point_on_consecutive_calls():
    import qdc_b200
    lib = qdc_b200.load()
    ctx = qdc_b200.context(0)
    cases = [  # (seed, n, hidden, vocab, with_add, dtype): a big call, then smaller ones
        (1, 3000, 1024, 151936, True, torch.float32),
        (2, 77, 1024, 4096, False, torch.float32),
        (3, 513, 1024, 8192, True, torch.bfloat16),
    ]
    for seed, n, hidden, vocab, with_add, dtype in cases:
        table, add, gamma, ids = _case(seed, n, hidden, vocab, with_add, dtype)
        x_new, y_new, x_ref, y_ref = (_nan(n, hidden, dtype) for _ in range(4))
        _noalloc(lib, x_new, y_new, table, add, gamma, ids)
        st = lib.qdc_gather_rms(ctx.handle, _vp(x_ref), _vp(y_ref), _vp(table),
                                ids.ctypes.data_as(ctypes.c_void_p), _vp(add), _vp(gamma), 1e-6, 1, n,
                                hidden, vocab, _code(dtype), _stream())
        assert st == 0, lib.qdc_last_error(ctx.handle)
        torch.cuda.synchronize()
        assert np.array_equal(_host(x_new), _host(x_ref))  # the gather itself is bit-exact
        rtol = 1e-5 if dtype == torch.float32 else 1e-2
        assert _close(_host(y_new), _host(y_ref), rtol)
        assert not np.isnan(_host(y_new)).any()


@pytest.mark.parametrize("hidden,dtype", [(768, torch.float32), (1024, torch.float32),
                                          (2048, torch.float32), (1000, torch.float32),
                                          (1024, torch.bfloat16), (1536, torch.bfloat16)])
def test_noalloc_matches_oracle(oracle, hidden, dtype):
    """Every row-kernel shape the entry point picks (vector kernels of 6, 8,
    16 Float32 chunks and 4, 6 bf16 chunks per lane; the scalar kernel for
    an odd width), two calls in a row, against the oracle."""
    import qdc_b200
    lib = qdc_b200.load()
    vocab = 3001
    for seed, n in ((11, 1200), (12, 33)):
        table, add, gamma, ids = _case(seed + hidden, n, hidden, vocab, True, dtype)
        x, y = _nan(n, hidden, dtype), _nan(n, hidden, dtype)
        _noalloc(lib, x, y, table, add, gamma, ids)
        torch.cuda.synchronize()
        g = gamma.cpu().numpy()
        if dtype == torch.float32:
            ex_x, ex_y = oracle.gather_rms(table.cpu().numpy(), ids, add.cpu().numpy(), g, 1e-6)
            assert np.array_equal(_host(x), ex_x)
            assert _close(_host(y), ex_y, 1e-5)
        else:
            bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
            ex_x, ex_y = oracle.gather_rms(bits(table), ids, bits(add), g, 1e-6)
            assert np.array_equal(bits(x), ex_x)
            assert _close(_host(y), oracle.bf16_decode(ex_y), 1e-2)


def test_noalloc_later_calls_take_no_device_memory():
    """After the first call on the device (which, under lazy module loading,
    brings the library's module and its fixed array onto the GPU), calls
    leave the device's free memory unchanged."""
    import qdc_b200
    lib = qdc_b200.load()
    table, add, gamma, ids = _case(21, 4096, 1024, 151936, True, torch.float32)
    x, y = _nan(4096, 1024, torch.float32), _nan(4096, 1024, torch.float32)
    _noalloc(lib, x, y, table, add, gamma, ids)
    torch.cuda.synchronize()
    free = []
    for _ in range(3):
        free.append(torch.cuda.mem_get_info()[0])
        _noalloc(lib, x, y, table, add, gamma, ids)
        torch.cuda.synchronize()
    free.append(torch.cuda.mem_get_info()[0])
    assert len(set(free)) == 1, free


def test_noalloc_rejects_oversize_and_bad_ids_before_launch():
    import qdc_b200
    lib = qdc_b200.load()
    table = torch.zeros((64, 1024), device="cuda")
    out = torch.zeros((8, 1024), device="cuda")
    gamma = torch.zeros((1024,), device="cuda")
    big = np.zeros(65537, np.int32)
    st = lib.qdc_gather_rms_noalloc(_vp(out), None, _vp(table), big.ctypes.data_as(ctypes.c_void_p),
                                    None, None, 1e-6, 1, big.size, 1024, 64, 0, _stream())
    assert st == qdc_b200._lib.QDC_EINVAL
    assert b"65536" in lib.qdc_last_error(None)
    bad = np.array([1, 64], np.int32)
    st = lib.qdc_gather_rms_noalloc(_vp(out), _vp(out), _vp(table), bad.ctypes.data_as(ctypes.c_void_p),
                                    None, _vp(gamma), 1e-6, 1, bad.size, 1024, 64, 0, _stream())
    assert st == qdc_b200._lib.QDC_EBOUNDS
    torch.cuda.synchronize()
