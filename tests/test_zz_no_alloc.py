"""qdc_gather_rms_noalloc -- the gather + input norm for callers that may not
allocate device memory (hosts whose memory pool owns every device byte,
loops that cannot take cudaMalloc's device-wide synchronisation, fixed
memory budgets).  It needs no context and keeps its id staging in a fixed
array inside the library.

Called here through the C ABI (ctypes) and compared with the context-based
entry point, qdc_gather_rms, on consecutive calls: the second call must not
see anything of the first (the shared array keeps the last call's contents).
This file sorts last so a stop-at-first-failure run has run everything else
first; it also passes alone in a fresh process."""
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


def _run(lib, ctx, table, add, gamma, ids, dtype):
    import qdc_b200
    n, hidden, vocab = ids.size, table.shape[1], table.shape[0]
    code = qdc_b200.QDC_F32 if dtype == torch.float32 else qdc_b200.QDC_BF16
    nan = lambda: torch.full((n, hidden), float("nan"), device="cuda").to(dtype)
    x_new, y_new, x_ref, y_ref = nan(), nan(), nan(), nan()
    host_ids = ids.ctypes.data_as(ctypes.c_void_p)
    st = lib.qdc_gather_rms_noalloc(_vp(x_new), _vp(y_new), _vp(table), host_ids, _vp(add),
                                    _vp(gamma), 1e-6, 1, n, hidden, vocab, code, _stream())
    assert st == 0, lib.qdc_last_error(None)
    st = lib.qdc_gather_rms(ctx.handle, _vp(x_ref), _vp(y_ref), _vp(table), host_ids, _vp(add),
                            _vp(gamma), 1e-6, 1, n, hidden, vocab, code, _stream())
    assert st == 0, lib.qdc_last_error(ctx.handle)
    torch.cuda.synchronize()
    return x_new.float().cpu().numpy(), y_new.float().cpu().numpy(), \
        x_ref.float().cpu().numpy(), y_ref.float().cpu().numpy()


def _close(a, b, rtol):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return bool((np.abs(a - b) <= 1e-6 + rtol * np.abs(b)).all())


def test_noalloc_matches_context_entry_point_on_consecutive_calls():
    import qdc_b200
    lib = qdc_b200.load()
    ctx = qdc_b200.context(0)
    cases = [  # (seed, n, hidden, vocab, with_add, dtype): a big call, then a smaller one
        (1, 3000, 1024, 151936, True, torch.float32),
        (2, 77, 1024, 4096, False, torch.float32),
        (3, 513, 1024, 8192, True, torch.bfloat16),
    ]
    for seed, n, hidden, vocab, with_add, dtype in cases:
        table, add, gamma, ids = _case(seed, n, hidden, vocab, with_add, dtype)
        x_new, y_new, x_ref, y_ref = _run(lib, ctx, table, add, gamma, ids, dtype)
        assert np.array_equal(x_new, x_ref)  # the gather itself is bit-exact
        rtol = 1e-5 if dtype == torch.float32 else 1e-2
        assert _close(y_new, y_ref, rtol)
        assert not np.isnan(y_new).any()


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
