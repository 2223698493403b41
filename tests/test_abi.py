"""The C-ABI library loads and exports every entry point include/qdc_b200.h
declares, and its host-only parts behave -- no GPU needed (no kernel is
launched here)."""
import ctypes

import numpy as np
import pytest


@pytest.fixture(scope="module")
def lib():
    import qdc_b200
    return qdc_b200.load()


def test_exports_every_declared_symbol(lib):
    import qdc_b200
    declared = qdc_b200.declared_symbols()
    assert len(declared) >= 18
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    from qdc_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared  # the binding covers the header exactly


def test_version_and_status_strings(lib):
    assert lib.qdc_abi_version() == 1
    assert lib.qdc_status_string(0) == b"ok"
    assert b"vocabulary" in lib.qdc_status_string(2)


def test_rope_table_matches_oracle_bit_for_bit(lib, oracle):
    import qdc_b200
    for theta, rotary, n in [(1e7, 64, 2048), (1e4, 4, 65), (1e7, 16, 300), (1e6, 128, 17)]:
        c, s = qdc_b200.rope_table(theta, rotary, n)
        oc, os_ = oracle.rope_table(theta, rotary, n)
        assert np.array_equal(c.numpy(), oc) and np.array_equal(s.numpy(), os_)


def test_rope_table_rejects_bad_arguments(lib):
    import qdc_b200
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.rope_table(1e4, 3, 4)  # odd rotary
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.rope_table(-1.0, 4, 4)


def test_null_context_is_rejected_without_touching_the_device(lib):
    # Every entry point checks its context first; nothing is launched.
    assert lib.qdc_residual_rms(None, None, None, None, None, None, 1e-6, 1, 1, 8, 8, 8, 8, 8, 0,
                                None) == 1
    assert lib.qdc_swiglu(None, None, None, None, None, 1, 4, 4, 4, 4, None) == 1
    assert lib.qdc_ws_alloc(None, 16, 256, ctypes.byref(ctypes.c_void_p())) == 1
    assert lib.qdc_set_option(None, 1, 0) == 1
    assert lib.qdc_bf16_to_f32(None, None, None, 8, None) == 1
    assert lib.qdc_f32_to_bf16(None, None, None, 8, None) == 1
    assert lib.qdc_delta_gates(None, None, None, None, 16, 0, None, None, 1, 4, None) == 1
    assert b"NULL" in lib.qdc_last_error(None)


def test_tensor_ops_refuse_cpu_tensors():
    import torch
    import qdc_b200
    x = torch.zeros(4, 8)
    w = torch.zeros(8)
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.native_rms(x, w, 1e-6)
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.native_mlp_gate(x, x)
