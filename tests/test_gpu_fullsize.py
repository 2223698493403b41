"""Parity at the full benchmark sizes (16,384-65,536 tokens of the 0.8B-shaped
backbone), kernel by kernel, against
the oracle run multi-threaded on the host.  Each case also exercises the
launch shape chosen for large unit counts."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q(oracle):
    import qdc_b200
    oracle.set_threads(os.cpu_count() or 1)
    yield qdc_b200
    oracle.set_threads(1)


def close(actual, expected, rtol=1e-5):
    a = actual.detach().float().cpu().numpy().astype(np.float64) if torch.is_tensor(actual) else actual
    e = np.asarray(expected, np.float64)
    return bool((np.abs(a - e) <= 1e-6 + rtol * np.abs(e)).all())


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_config2_gather_residual_rms(q, oracle):
    rng = np.random.default_rng(2)
    table = rng.standard_normal((151936, 1024), dtype=np.float32) * np.float32(0.02)
    ids = rng.integers(0, 151936, 16384).astype(np.int32)
    m = rng.standard_normal((16384, 1024), dtype=np.float32)
    w = rng.standard_normal(1024, dtype=np.float32) * np.float32(0.02)
    ex_r, ex_y = oracle.gather_rms(table, ids, m, w, 1e-6)
    x, y = q.native_gather_rms(dev(table), ids, dev(w), 1e-6, add=dev(m))
    assert np.array_equal(x.cpu().numpy(), ex_r) and close(y, ex_y)
    t16, m16 = oracle.bf16_encode(table), oracle.bf16_encode(m)
    ex_r16, ex_y16 = oracle.gather_rms(t16, ids, m16, w, 1e-6)
    b = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    x16, y16 = q.native_gather_rms(b(t16), ids, dev(w), 1e-6, add=b(m16))
    dec = lambda t: oracle.bf16_decode(t.cpu().view(torch.int16).numpy().view(np.uint16))
    assert close(dec(x16), oracle.bf16_decode(ex_r16), 1e-2)
    assert close(dec(y16), oracle.bf16_decode(ex_y16), 1e-2)


@pytest.mark.parametrize("tokens", [16384, 65536])
def test_config3_and_5_qk_norm_rope(q, oracle, tokens):
    rng = np.random.default_rng(tokens)
    proj = rng.standard_normal((tokens, 8 * 512 + 2 * 2 * 256), dtype=np.float32)
    qg = proj[:, :4096].reshape(tokens, 8, 512)
    kr = proj[:, 4096:4608].reshape(tokens, 2, 256)
    wq = rng.standard_normal(256, dtype=np.float32) * np.float32(0.02)
    wk = rng.standard_normal(256, dtype=np.float32) * np.float32(0.02)
    cos, sin = oracle.rope_table(1e7, 64, 2048)
    eq = oracle.qk_norm_rope(np.ascontiguousarray(qg[:, :, :256]), wq, 1e-6, 64, cos, sin, seq_len=2048)
    ek = oracle.qk_norm_rope(np.ascontiguousarray(kr), wk, 1e-6, 64, cos, sin, seq_len=2048)
    dp = dev(proj)
    dc, ds = q.rope_table(1e7, 64, 2048, device="cuda")
    gq, gk = q.native_q_k_norm_rope(dp[:, :4096].view(tokens, 8, 512)[:, :, :256],
                                    dp[:, 4096:4608].view(tokens, 2, 256), dev(wq), dev(wk), 1e-6, 64,
                                    dc, ds, seq_len=2048)
    assert close(gq, eq) and close(gk, ek)


def test_config4_residual_rms_and_swiglu(q, oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((32768, 1024), dtype=np.float32)
    m = rng.standard_normal((32768, 1024), dtype=np.float32)
    w = rng.standard_normal(1024, dtype=np.float32) * np.float32(0.02)
    ex_r, ex_y = oracle.residual_rms(x, m, w, 1e-6)
    r, y = q.native_residual_rms(dev(x), dev(m), dev(w), 1e-6)
    assert np.array_equal(r.cpu().numpy(), ex_r) and close(y, ex_y)
    del x, m, r, y
    g = rng.standard_normal((32768, 3584), dtype=np.float32)
    u = rng.standard_normal((32768, 3584), dtype=np.float32)
    e32, e16 = oracle.swiglu(g, u, want_bf16=True)
    h32, h16 = q.native_mlp_gate(dev(g), dev(u), want_bf16=True)
    assert close(h32, e32)
    dec = oracle.bf16_decode(h16.cpu().view(torch.int16).numpy().view(np.uint16))
    assert close(dec, oracle.bf16_decode(e16), 1e-2)


def test_config5_gated_rms(q, oracle):
    rng = np.random.default_rng(5)
    T = 65536
    o = rng.standard_normal((T, 16, 128), dtype=np.float32)
    proj = rng.standard_normal((T, 8224), dtype=np.float32)
    z = proj[:, 6144:8192].reshape(T, 16, 128)
    w = (1 + rng.standard_normal(128, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    expected = oracle.gated_rms(o, np.ascontiguousarray(z), w, 1e-6)
    dp = dev(proj)
    got = q.native_gated_rms(dev(o), dp[:, 6144:8192].view(T, 16, 128), dev(w), 1e-6)
    assert close(got, expected)


def test_0p8b_delta_conv_norm_48_heads(q, oracle):
    """The DeltaNet prologue at the 0.8B backbone's shape: 6,144 channels
    (16 q + 16 k + 16 v heads of 128) read in place from the packed
    [qkv | z | a | b] rows (8,224 wide), 32,768 tokens as 16 sequences of
    2,048 -- the shared-memory pipeline kernel."""
    rng = np.random.default_rng(6)
    T, C, W = 32768, 6144, 8224
    proj = rng.standard_normal((T, W), dtype=np.float32)
    conv = (rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    eq, ek, ev = oracle.delta_conv_norm(proj, conv, 16, 128, 16, 128, seq_len=2048)
    gq, gk, gv = q.native_delta_conv_norm(dev(proj), dev(conv), 16, 128, 16, 128, seq_len=2048)
    assert close(gq, eq) and close(gk, ek) and close(gv, ev)


def test_0p8b_attn_gate_8_heads_256(q, oracle):
    """The attention output gate at the 0.8B backbone's shape: values
    (16 sequences, 8 heads, 2048, 256) and the gate half of the packed
    [q;gate] projection (32,768 tokens x 8 x 512)."""
    rng = np.random.default_rng(7)
    B, H, S, D = 16, 8, 2048, 256
    values = rng.standard_normal((B, H, S, D), dtype=np.float32)
    qgate = rng.standard_normal((B * S, H, 2 * D), dtype=np.float32)
    expected = oracle.attn_gate(values, np.ascontiguousarray(qgate[:, :, D:]))
    got = q.native_attn_gate(dev(values), dev(qgate)[:, :, D:])
    assert close(got, expected)


def test_0p8b_delta_gates_16_heads(q, oracle):
    """The DeltaNet beta / decay gates at the 0.8B backbone's shape: a and b
    (16 heads each) read from the tail of the packed 8,224-wide projection
    rows, 65,536 tokens; inputs spread over [-30, 30] so the softplus and
    sigmoid reach both tails."""
    rng = np.random.default_rng(8)
    T, W, start = 65536, 8224, 6144 + 2048
    proj = rng.standard_normal((T, W), dtype=np.float32)
    proj[:, start:] = rng.uniform(-30, 30, (T, W - start)).astype(np.float32)
    a_decay = (-np.exp(rng.uniform(-1, 0.5, 16))).astype(np.float32)
    dt_bias = rng.standard_normal(16, dtype=np.float32)
    eb, ed = oracle.delta_gates(proj, start, 16, a_decay, dt_bias)
    gb, gd = q.native_delta_gates(dev(proj), start, 16, dev(a_decay), dev(dt_bias))
    assert close(gb, eb) and close(gd, ed)


def test_grid_stride_loops_past_the_grid_cap(q, oracle):
    """Grids stop where a loop's stride reaches 2^24 of the kernel's own
    units, and larger launches loop.  The DeltaNet gates count their units
    in 32 bits, one per thread: 2^24 + 4097 (token, head) units with one head
    take the cap of 65,536 blocks of 256 threads, so 4,097 threads take a
    second step of the grid-stride loop.  The residual
    norm (64-bit rows) at width 32 over 2^24 + 1,237 rows takes the
    4,194,304-block cap of its 4-row blocks; sampled rows are checked
    (first, around each multiple of the stride, last)."""
    rng = np.random.default_rng(24)
    tokens = (1 << 24) + 4097
    proj = rng.normal(0, 5, (tokens, 2)).astype(np.float32)
    a_decay = np.array([-0.7], np.float32)
    dt_bias = np.array([0.3], np.float32)
    eb, ed = oracle.delta_gates(proj, 0, 1, a_decay, dt_bias)
    gb, gd = q.native_delta_gates(dev(proj), 0, 1, dev(a_decay), dev(dt_bias))
    assert close(gb, eb) and close(gd, ed)
    del gb, gd, proj
    rows, width = (1 << 24) + 1237, 32
    g = torch.Generator(device="cuda")
    g.manual_seed(24)
    x = torch.randn((rows, width), generator=g, device="cuda")
    m = torch.randn((rows, width), generator=g, device="cuda")
    w = rng.normal(0, 0.02, width).astype(np.float32)
    r, y = q.native_residual_rms(x, m, dev(w), 1e-6)
    stride = (1 << 24) // 4 * 4  # rows per grid step: 4,194,304 blocks x 4 rows
    pick = np.unique(np.concatenate([np.arange(0, 64), np.arange(stride - 64, min(stride + 64, rows)),
                                     np.arange(rows - 64, rows),
                                     rng.integers(0, rows, 512)]))
    idx = torch.from_numpy(pick).cuda()
    xs, ms = x[idx].cpu().numpy(), m[idx].cpu().numpy()
    ex_r, ex_y = oracle.residual_rms(xs, ms, w, 1e-6)
    assert np.array_equal(r[idx].cpu().numpy(), ex_r) and close(y[idx], ex_y)


def test_residual_rms_bf16_32768_rows(q, oracle):
    """The bf16-stored residual norm at the MLP-norm size (32,768 x 1,024):
    r bit for bit against the oracle's integer rounding, y within 1e-2."""
    rng = np.random.default_rng(32)
    x = oracle.bf16_encode(rng.standard_normal((32768, 1024), dtype=np.float32))
    m = oracle.bf16_encode(rng.standard_normal((32768, 1024), dtype=np.float32))
    w = rng.standard_normal(1024, dtype=np.float32) * np.float32(0.02)
    ex_r, ex_y = oracle.residual_rms_bf16(x, m, w, 1e-6)
    b = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    r, y = q.native_residual_rms(b(x), b(m), dev(w), 1e-6)
    bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits(r), ex_r)
    assert close(oracle.bf16_decode(bits(y)), oracle.bf16_decode(ex_y), 1e-2)
