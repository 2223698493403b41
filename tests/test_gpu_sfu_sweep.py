"""Dense check of the SFU approximations against the oracle.

The Float32 kernels compute exp(-x) as ex2.approx(-x log2 e) and the
inverse as rcp.approx (SiLU in SwiGLU, in the gated norm and in the DeltaNet
conv; the sigmoid of the attention output gate), where the reference uses
IEEE exp and division (src/backbone.jl:196-197).  The argued bound is ~2 ulp
plus |x| * 6e-8 relative from rounding x log2 e.  Here EVERY Float32 of the
binades [2^-8, 2^-7), ..., [32, 64) and [64, 90], both signs, goes through
each of those kernels and is compared with the oracle (glibc expf and IEEE
division) at the kernel bar |a - b| <= 1e-6 + 1e-5 |b|."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-6, 1e-5
BINADES = list(range(-8, 7))  # [2^k, 2^(k+1)), the last one cut at 90


def binade(k):
    """Every Float32 in [2^k, min(2^(k+1), 90)], negative and positive."""
    lo = np.array([2.0 ** k], np.float32).view(np.uint32)[0]
    top = np.float32(90.0) if 2.0 ** (k + 1) > 90 else np.nextafter(np.float32(2.0 ** (k + 1)),
                                                                     np.float32(0))
    hi = np.array([top], np.float32).view(np.uint32)[0]
    x = np.arange(lo, hi + 1, dtype=np.uint32).view(np.float32)
    return np.concatenate([-x, x])


def padded(x, width):
    n = -(-x.size // width) * width
    out = np.zeros(n, np.float32)
    out[:x.size] = x
    return out.reshape(-1, width)


def assert_close(actual, expected, what):
    a = actual.detach().cpu().numpy().astype(np.float64) if torch.is_tensor(actual) else actual
    e = np.asarray(expected, np.float64)
    err = np.abs(a - e) - (ATOL + RTOL * np.abs(e))
    bad = err > 0
    assert not bad.any(), f"{what}: {int(bad.sum())} values outside the bar, worst at " \
                          f"expected {e.reshape(-1)[np.argmax(err)]!r}, got {a.reshape(-1)[np.argmax(err)]!r}"


@pytest.fixture(scope="module")
def q(oracle):
    import qdc_b200
    oracle.set_threads(os.cpu_count() or 1)
    yield qdc_b200
    oracle.set_threads(1)


@pytest.mark.parametrize("k", BINADES)
def test_silu_in_swiglu(q, oracle, k):
    g = padded(binade(k), 4096)
    u = np.ones_like(g)
    expected, _ = oracle.swiglu(g, u)
    got, _ = q.native_mlp_gate(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda())
    assert_close(got, expected, f"silu on [2^{k}, 2^{k + 1})")


@pytest.mark.parametrize("k", BINADES)
def test_sigmoid_in_attn_gate(q, oracle, k):
    gate = padded(binade(k), 8 * 256).reshape(-1, 8, 256)
    S = gate.shape[0]
    values = np.ones((1, 8, S, 256), np.float32)
    expected = oracle.attn_gate(values, gate)
    got = q.native_attn_gate(torch.from_numpy(values).cuda(), torch.from_numpy(gate).cuda())
    assert_close(got, expected, f"sigmoid on [2^{k}, 2^{k + 1})")


@pytest.mark.parametrize("k", BINADES)
def test_silu_in_gated_norm(q, oracle, k):
    z = padded(binade(k), 16 * 128).reshape(-1, 16, 128)
    o = np.ones_like(z)
    w = np.ones(128, np.float32)
    expected = oracle.gated_rms(o, z, w, 1e-6)
    got = q.native_gated_rms(torch.from_numpy(o).cuda(), torch.from_numpy(z).cuda(),
                             torch.from_numpy(w).cuda(), 1e-6)
    assert_close(got, expected, f"gated silu on [2^{k}, 2^{k + 1})")


@pytest.mark.parametrize("k", BINADES)
def test_silu_in_delta_conv(q, oracle, k):
    """The v channels of the DeltaNet prologue with conv taps (0, 0, 0, 1):
    v = silu(x) of the swept value (the shared-memory pipeline kernel:
    2 q + 2 k + 16 v heads of 128)."""
    kh, vh, d = 2, 16, 128
    v = padded(binade(k), vh * d)
    proj = np.zeros((v.shape[0], 2 * kh * d + vh * d), np.float32)
    proj[:, 2 * kh * d:] = v
    w = np.zeros((proj.shape[1], 4), np.float32)
    w[:, 3] = 1.0
    _, _, expected = oracle.delta_conv_norm(proj, w, kh, d, vh, d, seq_len=2048)
    _, _, got = q.native_delta_conv_norm(torch.from_numpy(proj).cuda(), torch.from_numpy(w).cuda(),
                                         kh, d, vh, d, seq_len=2048)
    assert_close(got, expected, f"conv silu on [2^{k}, 2^{k + 1})")
