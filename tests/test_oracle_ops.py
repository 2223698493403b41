"""Known-answer tests of the oracle's per-layer ops.

Cases follow the reference's own op tests: sin/cos ramps instead of random
data (test/backbone.jl:387-413 RMS widths 1/7/1024 x n 0/1/17; :354-385
rotary_dim 0/2/4; :741-760 gated output), checked against an independent
float64 numpy restatement at the reference's 2e-6 tolerance.
"""
import numpy as np
import pytest


def ramp(n, fn=np.sin):
    return fn(np.arange(1, n + 1, dtype=np.float32)).astype(np.float32)


def np_rms(x, w, eps, centered=True):
    x64 = x.astype(np.float64)
    scale = 1.0 / np.sqrt((x64 ** 2).sum(-1, keepdims=True) / x.shape[-1] + eps)
    g = (1.0 + w.astype(np.float64)) if centered else w.astype(np.float64)
    return x64 * scale * g


def close(a, b, tol=2e-6):
    return np.all(np.abs(np.asarray(a, np.float64) - b) <= tol + tol * np.abs(b))


@pytest.mark.parametrize("width", [1, 7, 1024])
@pytest.mark.parametrize("n", [0, 1, 17])
def test_rms_ramps(oracle, width, n):
    x = ramp(width * n).reshape(n, width)
    w = ramp(width, np.cos)
    saved = x.copy()
    y = oracle.rms(x, w, 1e-6)
    assert y.shape == (n, width)
    assert close(y, np_rms(x, w, 1e-6))
    assert np.array_equal(x, saved)
    assert close(oracle.rms(x, w, 1e-6, centered=False), np_rms(x, w, 1e-6, centered=False))


@pytest.mark.parametrize("width", [1, 7, 256, 1024])
def test_residual_rms(oracle, width):
    n = 17
    x = ramp(width * n).reshape(n, width)
    m = ramp(width * n, np.cos).reshape(n, width)
    w = ramp(width, np.cos) * np.float32(0.02)
    r, y = oracle.residual_rms(x, m, w, 1e-6)
    assert np.array_equal(r, (x + m).astype(np.float32))
    assert close(y, np_rms(x + m, w, 1e-6))
    r2, y2 = oracle.residual_rms(x, None, w, 1e-6, store_residual=False)
    assert r2 is None and close(y2, np_rms(x, w, 1e-6))


def test_zero_rows_scale_is_eps(oracle):
    x = np.zeros((3, 8), np.float32)
    w = np.zeros(8, np.float32)
    y = oracle.rms(x, w, 1e-6)
    assert np.array_equal(y, np.zeros_like(x))


def test_gather_bit_exact_and_bounds(oracle):
    table = ramp(64 * 8).reshape(64, 8)
    ids = np.array([3, 0, 63, 3], np.int32)
    assert np.array_equal(oracle.gather(table, ids), table[ids])
    with pytest.raises(IndexError):
        oracle.gather(table, np.array([64], np.int32))
    with pytest.raises(IndexError):
        oracle.gather(table, np.array([-1], np.int32))
    t16 = oracle.bf16_encode(table)
    assert np.array_equal(oracle.gather(t16, ids), t16[ids])


def test_bf16_convention(oracle):
    # src/safetensors.jl:38-42: RNE by integer add; ties to even
    vals = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0, -0.0, np.inf], np.float32)
    bits = oracle.bf16_encode(vals)
    assert list(bits) == [0x3F80, 0x3F80, 0x3F82, 0xC020, 0x0000, 0x8000, 0x7F80]
    assert np.array_equal(oracle.bf16_decode(bits)[:6], np.array([1, 1, 1.015625, -2.5, 0, -0.0], np.float32))
    # the formula has no NaN special case: 0x7fffffff wraps to 0x8000 (-0.0)
    assert int(oracle.bf16_encode(np.array([0x7FFFFFFF], np.uint32).view(np.float32))[0]) == 0x8000


def np_rope_table(theta, rotary, n):
    half = rotary // 2
    cos = np.empty((n, half), np.float32)
    sin = np.empty((n, half), np.float32)
    for j in range(half):
        e = np.float32(2 * j) / np.float32(rotary)
        freq = np.float32(1.0) / np.float32(np.float64(theta) ** np.float64(e))
        ang = (freq * np.arange(n, dtype=np.float32)).astype(np.float32)
        cos[:, j] = np.cos(ang.astype(np.float64)).astype(np.float32)
        sin[:, j] = np.sin(ang.astype(np.float64)).astype(np.float32)
    return cos, sin


@pytest.mark.parametrize("theta,rotary,n", [(1e4, 4, 65), (1e7, 64, 2048), (1e7, 16, 64), (1e4, 0, 3)])
def test_rope_table(oracle, theta, rotary, n):
    c, s = oracle.rope_table(theta, rotary, n)
    ec, es = np_rope_table(np.float32(theta), rotary, n)
    assert np.array_equal(c, ec) and np.array_equal(s, es)


@pytest.mark.parametrize("rotary", [0, 2, 4])
@pytest.mark.parametrize("n", [1, 17, 65])
def test_qk_norm_rope_ramps(oracle, rotary, n):
    heads, dim = 2, 4
    packed = ramp(n * heads * 2 * dim).reshape(n, heads, 2 * dim)
    w = ramp(dim, np.cos)
    c, s = oracle.rope_table(1e4, rotary, n)
    out = oracle.qk_norm_rope(packed[:, :, :dim], w, 1e-6, rotary, c, s)
    exp = np_rms(packed[:, :, :dim], w, 1e-6)
    half = rotary // 2
    a, b = exp[..., :half].copy(), exp[..., half:2 * half].copy()
    cc, ss = c[:, None, :].astype(np.float64), s[:, None, :].astype(np.float64)
    exp[..., :half] = a * cc - b * ss
    exp[..., half:2 * half] = b * cc + a * ss
    assert close(out, exp)


def test_qk_positions_offset_and_period(oracle):
    n, heads, dim, rotary = 12, 2, 8, 4
    x = ramp(n * heads * dim).reshape(n, heads, dim)
    w = np.zeros(dim, np.float32)
    c, s = oracle.rope_table(1e4, rotary, 10)
    # positions restart every seq_len tokens
    per = oracle.qk_norm_rope(x, w, 1e-6, rotary, c, s, seq_len=4)
    for t in range(n):
        one = oracle.qk_norm_rope(x[t:t + 1], w, 1e-6, rotary, c, s, pos_offset=t % 4)
        assert np.array_equal(per[t], one[0])


@pytest.mark.parametrize("n", [1, 17, 129])
def test_gated_rms_ramps(oracle, n):
    # test/backbone.jl:741-760 (width 128, 4 heads; z already activated there)
    width, heads = 128, 4
    raw = ramp(width * heads * n).reshape(n, heads, width)
    zraw = ramp(width * heads * n, np.cos).reshape(n, heads, width)
    w = ramp(width, np.cos)
    out = oracle.gated_rms(raw, zraw, w, 1e-6)
    z64 = zraw.astype(np.float64)
    exp = np_rms(raw, w, 1e-6, centered=False) * (z64 / (1 + np.exp(-z64)))
    assert close(out.reshape(n, heads, width), exp, 2e-5)


def test_swiglu_and_silu_edges(oracle):
    g = np.array([[0.0, -0.0, 1.0, -1.0, 30.0, -30.0, 100.0, -100.0, np.inf]], np.float32)
    u = np.full_like(g, 2.0)
    h, h16 = oracle.swiglu(g, u, want_bf16=True)
    g64 = g.astype(np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        exp = g64 / (1 + np.exp(-g64)) * 2.0
    assert close(h[:, :8], exp[:, :8])
    assert np.signbit(h[0, 1])  # -0 * 0.5 * 2 keeps its sign
    assert h[0, 8] == np.inf
    assert np.array_equal(h16, oracle.bf16_encode(h))
    # silu(-inf) = -inf * inv(1 + inf) = NaN, as the reference formula gives
    assert np.isnan(oracle.silu(np.array([-np.inf], np.float32)))[0]


def test_delta_gates_edges_and_packed_layout(oracle):
    """beta = inv(1 + exp(-b)), decay = a_decay * (max(x, 0) + log1p(exp(-|x|)))
    with x = a + dt_bias (src/backbone.jl:196-198, :292-297), a and b read
    from the tail of packed projection rows."""
    heads = 5
    edge = np.array([0.0, 1.0, -1.0, 30.0, -30.0, 100.0, -100.0, 0.5, -0.25, 7.0], np.float32)
    a = np.stack([edge[(np.arange(heads) + t) % edge.size] for t in range(6)])
    b = -a[:, ::-1].copy()
    lead = 9
    proj = np.concatenate([ramp(6 * lead).reshape(6, lead), a, b, np.ones((6, 3), np.float32)], axis=1)
    proj = proj.astype(np.float32)
    a_decay = -np.exp(ramp(heads, np.cos)).astype(np.float32)
    dt_bias = (0.1 * ramp(heads)).astype(np.float32)
    beta, decay = oracle.delta_gates(proj, lead, heads, a_decay, dt_bias)
    x = a.astype(np.float64) + dt_bias.astype(np.float64)
    sp = np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))
    assert close(beta, 1.0 / (1.0 + np.exp(-b.astype(np.float64))))
    assert close(decay, a_decay.astype(np.float64) * sp)
    assert beta.shape == decay.shape == (6, heads)
    empty = oracle.delta_gates(proj[:0], lead, heads, a_decay, dt_bias)
    assert empty[0].shape == (0, heads)


def test_swiglu_packed_layout(oracle):
    rows, width = 5, 16
    packed = ramp(rows * 2 * width).reshape(rows, 2 * width)
    h, _ = oracle.swiglu(packed[:, :width], packed[:, width:])
    g = packed[:, :width].astype(np.float64)
    assert close(h, g / (1 + np.exp(-g)) * packed[:, width:])


def test_threads_do_not_change_results(oracle):
    x = ramp(300 * 256).reshape(300, 256)
    m = ramp(300 * 256, np.cos).reshape(300, 256)
    w = ramp(256)
    oracle.set_threads(1)
    a = oracle.residual_rms(x, m, w, 1e-6)
    oracle.set_threads(4)
    b = oracle.residual_rms(x, m, w, 1e-6)
    oracle.set_threads(1)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def _np_delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len, eps=1e-6):
    """float64 restatement: 4-tap causal conv (taps oldest first, absent
    before the sequence start), SiLU, per-head L2 norm of q (also / sqrt(kd))
    and k; v only activated (src/backbone_cpu.jl:787-807, :411-427)."""
    T = proj.shape[0]
    C = 2 * kh * kd + vh * vd
    x = proj[:, :C].astype(np.float64)
    conv = np.zeros((T, C))
    for t in range(T):
        pos = t % seq_len
        for j in range(4):
            if pos - 3 + j >= 0:
                conv[t] += x[t - 3 + j] * w[:, j]
    s = conv / (1.0 + np.exp(-conv))
    q = s[:, :kh * kd].reshape(T, kh, kd)
    k = s[:, kh * kd:2 * kh * kd].reshape(T, kh, kd)
    v = s[:, 2 * kh * kd:].reshape(T, vh, vd)
    nq = q / (np.sqrt((q ** 2).sum(-1, keepdims=True) + eps) * np.sqrt(kd))
    nk = k / np.sqrt((k ** 2).sum(-1, keepdims=True) + eps)
    return nq, nk, v


@pytest.mark.parametrize("tokens,seq_len", [(1, 1), (9, 4), (17, 17), (40, 13)])
def test_delta_conv_norm_ramps(oracle, tokens, seq_len):
    kh, kd, vh, vd = 2, 8, 3, 4
    C = 2 * kh * kd + vh * vd
    proj = ramp(tokens * (C + 5)).reshape(tokens, C + 5)
    w = (0.5 * ramp(C * 4, np.cos)).reshape(C, 4)
    gq, gk, gv = oracle.delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len=seq_len)
    eq, ek, ev = _np_delta_conv_norm(proj, w.astype(np.float64), kh, kd, vh, vd, seq_len)
    assert close(gq, eq) and close(gk, ek) and close(gv, ev)


def test_delta_conv_norm_edge_values(oracle):
    """The L2-norm edge values of test/backbone.jl:290-313 after an identity
    conv (each token its own sequence): exact results."""
    edges = np.array([0.0, -0.0, np.nan, np.inf, np.finfo(np.float32).max, 1e-45], np.float32)
    kh, kd, vh, vd = 1, 8, 1, 8
    C = 2 * kh * kd + vh * vd
    proj = np.repeat(edges[:, None], C, axis=1)
    w = np.zeros((C, 4), np.float32)
    w[:, 3] = 1.0
    q, k, v = oracle.delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len=1)
    big = np.finfo(np.float32).max
    # the conv accumulates into a +0 (value = 0; value += x * w, src/backbone_cpu.jl:
    # 787-807), so -0 comes out as +0; Inf normalises to inf/inf = NaN, floatmax
    # to max/inf = 0 (its square overflows the Float32 sum)
    expect_qk = np.array([0.0, 0.0, np.nan, np.nan, 0.0, 0.0], np.float32)
    expect_v = np.array([0.0, 0.0, np.nan, np.inf, big, 0.0], np.float32)    # silu only
    for got, exp in ((q, expect_qk), (k, expect_qk), (v, expect_v)):
        g = got.reshape(6, -1)
        for t in range(6):
            assert np.array_equal(g[t], np.full(g.shape[1], exp[t]), equal_nan=True), (t, g[t])
            if not np.isnan(exp[t]):  # a NaN's sign carries nothing
                assert np.array_equal(np.signbit(g[t]), np.full(g.shape[1], np.signbit(exp[t])))


@pytest.mark.parametrize("B,S,H,D", [(1, 1, 1, 4), (2, 5, 3, 8), (3, 7, 2, 16)])
def test_attn_gate_ramps(oracle, B, S, H, D):
    """values .* inv(1 + exp(-gate)), src/backbone.jl:258-259, with the
    attention output read in (B, H, S, D) and the gate in (B*S, H, D)."""
    values = ramp(B * H * S * D).reshape(B, H, S, D)
    packed = (3 * ramp(B * S * H * 2 * D, np.cos)).reshape(B * S, H, 2 * D)
    gate = packed[:, :, D:]
    got = oracle.attn_gate(values, np.ascontiguousarray(gate))
    v = values.astype(np.float64).transpose(0, 2, 1, 3).reshape(B * S, H, D)
    exp = v / (1.0 + np.exp(-gate.astype(np.float64)))
    assert close(got.reshape(B * S, H, D), exp)


def test_unit_lower_solve_matches_float64(oracle):
    """The oracle's delta_solve (forward substitution in Float32) against a
    float64 solve with the unit lower triangle of the same matrices."""
    rng = np.random.default_rng(3)
    for n, width in ((64, 256), (17, 3), (1, 4)):
        L = rng.uniform(-0.3, 0.3, (4, n, n)).astype(np.float32)
        L += np.triu(np.full((n, n), 9.0, np.float32))  # never read
        R = rng.standard_normal((4, n, width)).astype(np.float32)
        x = oracle.unit_lower_solve(L, R)
        exact = np.linalg.solve(np.tril(L.astype(np.float64), -1) + np.eye(n), R.astype(np.float64))
        assert np.all(np.abs(x - exact) <= 1e-5 * np.abs(exact).max(axis=1, keepdims=True) + 1e-6)
