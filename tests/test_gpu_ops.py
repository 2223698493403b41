"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Bar: the gather bit-exact; Float32 outputs within |a - b| <= 1e-6 + 1e-5 |b|;
bf16-stored outputs within 1e-2 relative.  Cases follow the reference's op
tests (odd widths 1/7, rows 0/1/17, rotary 0/2/4, packed projection
layouts, NaN-filled outputs that must be overwritten, inputs unchanged) plus
the 0.8B-shaped backbone's shapes (hidden 1024, head_dim 256 / rotary 64, Dv 128,
intermediate 3584).
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-6, 1e-5
BF16_RTOL = 1e-2


def f32_close(actual, expected):
    a = actual.detach().cpu().numpy().astype(np.float64) if torch.is_tensor(actual) else actual
    e = np.asarray(expected, np.float64)
    with np.errstate(invalid="ignore"):
        ok = np.abs(a - e) <= ATOL + RTOL * np.abs(e)
    ok |= (np.isnan(a) & np.isnan(e)) | (a == e)  # NaN matches NaN; equal infinities match
    return bool(ok.all())


def bf16_close(actual_bf16, expected_bits, oracle):
    a = actual_bf16.detach().cpu().view(torch.int16).numpy().view(np.uint16)
    av = oracle.bf16_decode(a).astype(np.float64)
    ev = oracle.bf16_decode(expected_bits).astype(np.float64)
    return bool((np.abs(av - ev) <= 1e-6 + BF16_RTOL * np.abs(ev)).all())


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def nan_like(shape, dtype=torch.float32):
    return torch.full(shape, float("nan"), dtype=dtype, device="cuda")


@pytest.fixture(scope="module")
def q():
    import qdc_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return qdc_b200


def rng(seed=0):
    return np.random.default_rng(seed)


# --------------------------------------------------------------- gather

@pytest.mark.parametrize("hidden", [1024, 256, 8, 1000])
@pytest.mark.parametrize("n", [0, 1, 17, 513])
def test_gather_bit_exact(q, oracle, hidden, n):
    r = rng(hidden + n)
    table = r.normal(0, 0.02, (4096, hidden)).astype(np.float32)
    ids = r.integers(0, 4096, n).astype(np.int32)
    out = q.native_gather(dev(table), ids)
    assert out.shape == (n, hidden)
    assert np.array_equal(out.cpu().numpy(), oracle.gather(table, ids))
    # bf16 table: bit-exact copy of the stored bits
    t16 = oracle.bf16_encode(table)
    out16 = q.native_gather(dev_bf16(t16), ids)
    assert np.array_equal(out16.cpu().view(torch.int16).numpy().view(np.uint16), t16[ids])


def test_gather_rejects_out_of_vocab_before_launch(q):
    table = dev(np.zeros((64, 8), np.float32))
    with pytest.raises(q.ArgumentError):
        q.native_gather(table, [1, 64])
    with pytest.raises(q.ArgumentError):
        q.native_gather(table, [-1])


def test_gather_device_ids_flag(q, oracle):
    table = rng(1).normal(0, 1, (64, 256)).astype(np.float32)
    ids = np.array([5, 64, 7, -3], np.int32)
    ctx = q.context(0)
    out = q.native_gather(dev(table), dev(ids), ctx=ctx)
    with pytest.raises(q.ArgumentError):
        ctx.sync()
    o = out.cpu().numpy()
    assert np.array_equal(o[0], table[5]) and np.array_equal(o[2], table[7])
    assert np.isnan(o[1]).all() and np.isnan(o[3]).all()
    ctx.sync()  # flag cleared by the previous report


@pytest.mark.parametrize("hidden", [1024, 256, 7])
@pytest.mark.parametrize("with_add", [False, True])
@pytest.mark.parametrize("centered", [True, False])
def test_gather_rms_f32(q, oracle, hidden, with_add, centered):
    r = rng(hidden)
    n, vocab = 77, 5000
    table = r.normal(0, 0.02, (vocab, hidden)).astype(np.float32)
    ids = r.integers(0, vocab, n).astype(np.int32)
    add = r.normal(0, 1, (n, hidden)).astype(np.float32) if with_add else None
    w = r.normal(0, 0.02, hidden).astype(np.float32)
    ex_r, ex_y = oracle.gather_rms(table, ids, add, w, 1e-6, centered)
    out_x, out_y = nan_like((n, hidden)), nan_like((n, hidden))
    x, y = q.native_gather_rms(dev(table), ids, dev(w), 1e-6, add=None if add is None else dev(add),
                               centered=centered, out_x=out_x, out_y=out_y)
    assert np.array_equal(x.cpu().numpy(), ex_r)  # r = E[id] + add: one Float32 add, exact
    assert f32_close(y, ex_y)


@pytest.mark.parametrize("hidden", [1024, 512, 24])
def test_gather_rms_bf16(q, oracle, hidden):
    r = rng(7)
    n, vocab = 300, 3000
    table = oracle.bf16_encode(r.normal(0, 0.02, (vocab, hidden)).astype(np.float32))
    add = oracle.bf16_encode(r.normal(0, 1, (n, hidden)).astype(np.float32))
    ids = r.integers(0, vocab, n).astype(np.int32)
    w = r.normal(0, 0.02, hidden).astype(np.float32)
    ex_r, ex_y = oracle.gather_rms(table, ids, add, w, 1e-6)
    x, y = q.native_gather_rms(dev_bf16(table), ids, dev(w), 1e-6, add=dev_bf16(add))
    assert bf16_close(x, ex_r, oracle) and bf16_close(y, ex_y, oracle)


# ---------------------------------------------------------- residual RMS

@pytest.mark.parametrize("width", [1, 7, 128, 256, 768, 1024, 2048, 1000, 4096])
@pytest.mark.parametrize("rows", [0, 1, 17, 300])
def test_residual_rms_f32(q, oracle, width, rows):
    r = rng(width * 1000 + rows)
    x = r.normal(0, 1, (rows, width)).astype(np.float32)
    m = r.normal(0, 1, (rows, width)).astype(np.float32)
    w = r.normal(0, 0.02, width).astype(np.float32)
    ex_r, ex_y = oracle.residual_rms(x, m, w, 1e-6)
    dx, dm = dev(x), dev(m)
    out_r, out_y = nan_like((rows, width)), nan_like((rows, width))
    res, y = q.native_residual_rms(dx, dm, dev(w), 1e-6, out_r=out_r, out_y=out_y)
    assert np.array_equal(res.cpu().numpy(), ex_r)
    assert f32_close(y, ex_y)
    assert np.array_equal(dx.cpu().numpy(), x) and np.array_equal(dm.cpu().numpy(), m)
    # plain RMSNorm (input / final norm), centered and not
    for centered in (True, False):
        y2 = q.native_rms(dx, dev(w), 1e-6, centered=centered)
        assert f32_close(y2, oracle.rms(x, w, 1e-6, centered=centered))


def test_residual_rms_in_place_and_strided(q, oracle):
    r = rng(3)
    rows, width, ld = 65, 1024, 1536
    big = r.normal(0, 1, (rows, ld)).astype(np.float32)
    m = r.normal(0, 1, (rows, width)).astype(np.float32)
    w = r.normal(0, 0.02, width).astype(np.float32)
    ex_r, ex_y = oracle.residual_rms(big[:, :width], m, w, 1e-6)
    dbig = dev(big)
    view = dbig[:, :width]
    res, y = q.native_residual_add_rms(view, dev(m), dev(w), 1e-6)
    assert res.data_ptr() == view.data_ptr()
    got = dbig.cpu().numpy()
    assert np.array_equal(got[:, :width], ex_r)
    assert np.array_equal(got[:, width:], big[:, width:])  # padding untouched
    assert f32_close(y, ex_y)


@pytest.mark.parametrize("width", [1024, 256, 40])
def test_residual_rms_bf16(q, oracle, width):
    r = rng(width)
    rows = 129
    x = oracle.bf16_encode(r.normal(0, 1, (rows, width)).astype(np.float32))
    m = oracle.bf16_encode(r.normal(0, 1, (rows, width)).astype(np.float32))
    w = r.normal(0, 0.02, width).astype(np.float32)
    ex_r, ex_y = oracle.residual_rms_bf16(x, m, w, 1e-6)
    res, y = q.native_residual_rms(dev_bf16(x), dev_bf16(m), dev(w), 1e-6)
    assert bf16_close(res, ex_r, oracle) and bf16_close(y, ex_y, oracle)


def _bf16_bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def _f32_patterns(r, n):
    """Float32 values that stress rounding to bf16: exact ties (low half
    0x8000) on odd and even bf16 mantissas, one below and above a tie,
    carries into the exponent, subnormals, the largest finites (overflow
    to infinity), infinities, both signs, and random bit patterns."""
    hi = r.integers(0, 0x7f80, n).astype(np.uint32) << 16
    low = r.choice(np.array([0x8000, 0x7fff, 0x8001, 0xffff, 0x0000], np.uint32), n)
    low = np.where(r.random(n) < 0.3, r.integers(0, 0x10000, n).astype(np.uint32), low)
    bits = hi | low
    k = n // 8
    bits[:k] = r.integers(1, 0x800000, k).astype(np.uint32)  # subnormals
    bits[k:k + 16] = 0x7f7fffff - np.arange(16, dtype=np.uint32) * 0x1000  # near the largest finite
    bits[k + 16] = 0x7f800000  # infinity
    bits |= (r.random(n) < 0.5).astype(np.uint32) << 31
    return bits.view(np.float32)


def test_bf16_row_store_rounding_is_bit_exact(q, oracle):
    """The bf16 row kernel rounds its results by the reference's integer
    rounding (src/safetensors.jl:38-42), and rows whose results may hold a
    NaN (a non-finite sum of squares or scale) by the hardware conversion,
    so that a NaN result stays a NaN (the integer rounding of the GPU's
    canonical NaN would store -0.0).  Both must give the integer rounding's
    bits for every value that is not a NaN.  A gathered row with no add is
    copied bit for bit, NaN payloads included.

    r = x + m over bf16 pairs a few exponents apart, so the Float32 sum has
    bits below bf16 precision (ties, carries), checked bit for bit; one row
    holds a NaN.  y: rows of r = +1 and -1 with eps 0 give a scale of
    exactly 1, so y = +-gamma, and gamma runs over `_f32_patterns`
    (subnormals, ties, overflow); a zero row beside them has an infinite
    scale, so its y is NaN."""
    r = rng(77)
    rows, width = 512, 1024
    xb = r.integers(0x0080, 0x7f00, (rows, width)).astype(np.uint16)
    shift = r.integers(1, 12, (rows, width)).astype(np.uint16) << 7  # 1-11 binades lower
    mb = np.where(xb > shift + 0x0080, xb - shift, xb).astype(np.uint16)
    xb |= (r.random((rows, width)) < 0.5).astype(np.uint16) << 15
    mb |= (r.random((rows, width)) < 0.5).astype(np.uint16) << 15
    xb[0, :4] = [0x3f80, 0x3f81, 0xbf80, 0x3f80]  # 1 + 2^-8 and friends: exact ties
    mb[0, :4] = [0x3b80, 0x3b80, 0xbb80, 0x3c00]
    xb[1, 7] = 0x7fc0  # a NaN in row 1
    w = r.normal(0, 0.02, width).astype(np.float32)
    res, _ = q.native_residual_rms(dev_bf16(xb), dev_bf16(mb), dev(w), 1e-6)
    exact = oracle.bf16_decode(xb) + oracle.bf16_decode(mb)  # IEEE Float32 sums
    expected = oracle.bf16_encode(exact)
    got = _bf16_bits(res)
    keep = ~np.isnan(exact)
    assert np.array_equal(got[keep], expected[keep])
    assert np.isnan(oracle.bf16_decode(got[1, 7:8])).all()
    ones = np.zeros((3, width), np.uint16)
    ones[0], ones[1] = 0x3f80, 0xbf80  # rows of +1 and -1; row 2 stays zero
    for launch in range(16):
        g = _f32_patterns(rng(100 + launch), width)
        _, y = q.native_residual_rms(dev_bf16(ones), None, dev(g), 0.0, centered=False)
        got = _bf16_bits(y)
        for row, sign in ((0, 1.0), (1, -1.0)):
            want = oracle.bf16_encode((np.float32(sign) * g).astype(np.float32))
            assert np.array_equal(got[row], want), (launch, row)
        assert np.isnan(oracle.bf16_decode(got[2])).all()  # 0 x inf
    # the scalar kernel (width 40) rounds per value: the same bits, NaN kept
    xs, ms = xb[:64, :40].copy(), mb[:64, :40].copy()
    xs[5, 3] = 0xffc1  # a NaN
    res40, _ = q.native_residual_rms(dev_bf16(xs), dev_bf16(ms), dev(w[:40]), 1e-6)
    exact40 = oracle.bf16_decode(xs) + oracle.bf16_decode(ms)
    got40 = _bf16_bits(res40)
    keep40 = ~np.isnan(exact40)
    assert np.array_equal(got40[keep40], oracle.bf16_encode(exact40)[keep40])
    assert np.isnan(oracle.bf16_decode(got40[~keep40])).all()
    # the gather alone: the table's words, NaN payloads and -0 included
    table = r.integers(0, 0x10000, (64, width)).astype(np.uint16)
    table[3, :4] = [0x7fc1, 0xffff, 0x7f81, 0x8000]
    ids = np.array([3, 0, 63, 3, 17], np.int32)
    x, _ = q.native_gather_rms(dev_bf16(table), ids, dev(w), 1e-6)
    assert np.array_equal(_bf16_bits(x), table[ids])


def test_rms_edge_values(q, oracle):
    x = np.zeros((4, 1024), np.float32)
    x[1] = 1e-30
    x[2, :3] = np.float32(3e38)  # overflowing sum of squares -> scale 0
    x[3] = np.nan
    w = np.zeros(1024, np.float32)
    y = q.native_rms(dev(x), dev(w), 1e-6)
    assert f32_close(y, oracle.rms(x, w, 1e-6))


def test_residual_rms_validation(q):
    x = torch.zeros(4, 8, device="cuda")
    with pytest.raises(q.DimensionMismatch):
        q.native_residual_rms(x, torch.zeros(4, 9, device="cuda"), torch.zeros(8, device="cuda"), 1e-6)
    with pytest.raises(q.DimensionMismatch):
        q.native_rms(x, torch.zeros(7, device="cuda"), 1e-6)


# ----------------------------------------------------------- q/k norm + RoPE

QK_CASES = [  # tokens, heads, dim, rotary, packed (q inside a [q;gate] projection)
    (17, 8, 256, 64, True), (33, 2, 256, 64, False), (40, 4, 64, 16, True), (9, 2, 4, 4, True),
    (9, 2, 4, 2, False), (9, 1, 4, 0, False), (13, 3, 128, 128, False), (7, 2, 96, 32, True),
    (5, 2, 256, 256, False), (1, 8, 256, 64, True), (0, 8, 256, 64, True), (21, 2, 512, 64, False),
    (11, 2, 32, 8, False),
]


@pytest.mark.parametrize("tokens,heads,dim,rotary,packed", QK_CASES)
def test_qk_norm_rope(q, oracle, tokens, heads, dim, rotary, packed):
    r = rng(tokens * 31 + dim + rotary)
    width = 2 * dim if packed else dim
    proj = r.normal(0, 1, (tokens, heads, width)).astype(np.float32)
    w = r.normal(0, 0.02, dim).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, rotary, max(tokens, 1))
    expected = oracle.qk_norm_rope(proj[:, :, :dim], w, 1e-6, rotary, cos, sin)
    dproj = dev(proj)
    out = nan_like((tokens, heads, dim))
    dc, ds = q.rope_table(1e7, rotary, max(tokens, 1), device="cuda")
    got = q.native_qk_norm_rope(dproj[:, :, :dim], dev(w), 1e-6, rotary, dc, ds, out=out)
    assert f32_close(got, expected)
    assert np.array_equal(dproj.cpu().numpy(), proj)


def test_qk_positions_sequence_sharded(q, oracle):
    """pos = offset + t mod seq_len: sequences packed back to back (the
    multi-GPU shard layout) and the final-query offset of
    src/backbone_cpu.jl:1012-1016."""
    r = rng(11)
    seqs, seq_len, heads, dim, rotary = 3, 50, 2, 256, 64
    x = r.normal(0, 1, (seqs * seq_len, heads, dim)).astype(np.float32)
    w = r.normal(0, 0.02, dim).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, rotary, 2048)
    dc, ds = q.rope_table(1e7, rotary, 2048, device="cuda")
    got = q.native_qk_norm_rope(dev(x), dev(w), 1e-6, rotary, dc, ds, seq_len=seq_len)
    for s in range(seqs):
        sl = slice(s * seq_len, (s + 1) * seq_len)
        assert f32_close(got[sl], oracle.qk_norm_rope(x[sl], w, 1e-6, rotary, cos, sin))
    last = q.native_qk_norm_rope(dev(x[-1:]), dev(w), 1e-6, rotary, dc, ds, pos_offset=2047)
    assert f32_close(last, oracle.qk_norm_rope(x[-1:], w, 1e-6, rotary, cos, sin, pos_offset=2047))
    with pytest.raises(q.ArgumentError):  # beyond the table
        q.native_qk_norm_rope(dev(x[-2:]), dev(w), 1e-6, rotary, dc, ds, pos_offset=2047)


# --------------------------------------------------------------- gated RMS

GATED_CASES = [(17, 16, 128), (5, 4, 128), (9, 2, 2), (33, 3, 64), (1, 16, 128), (0, 16, 128),
               (12, 2, 256), (7, 5, 48)]


@pytest.mark.parametrize("rows,heads,dim", GATED_CASES)
def test_gated_rms(q, oracle, rows, heads, dim):
    r = rng(rows + heads + dim)
    o = r.normal(0, 1, (rows, heads, dim)).astype(np.float32)
    # z lives inside a packed [qkv | z | a | b] projection row
    lead, tail = 3 * dim * heads + (4 if dim % 4 == 0 else 1), 8
    packed = r.normal(0, 1, (rows, lead + heads * dim + tail)).astype(np.float32)
    z = packed[:, lead:lead + heads * dim].reshape(rows, heads, dim)
    w = (1 + r.normal(0, 0.02, dim)).astype(np.float32)
    expected = oracle.gated_rms(o, np.ascontiguousarray(z), w, 1e-6)
    dpacked = dev(packed)
    dz = dpacked[:, lead:lead + heads * dim].view(rows, heads, dim) if rows else \
        torch.empty((0, heads, dim), device="cuda")
    got = q.native_gated_rms(dev(o), dz, dev(w), 1e-6, out=nan_like((rows, heads * dim)))
    assert f32_close(got, expected)


# ------------------------------------------------------------------ SwiGLU

@pytest.mark.parametrize("rows,width", [(17, 3584), (3, 768), (5, 16), (7, 13), (1, 4), (0, 64),
                                        (33, 1000)])
@pytest.mark.parametrize("packed", [True, False])
def test_swiglu(q, oracle, rows, width, packed):
    r = rng(rows * width)
    if packed:  # [gate | up] per token, ext/cuda_mlp.jl:63-71
        proj = r.normal(0, 1, (rows, 2 * width)).astype(np.float32)
        g, u = proj[:, :width], proj[:, width:]
        dproj = dev(proj)
        dg, du = dproj[:, :width], dproj[:, width:]
    else:
        g = r.normal(0, 1, (rows, width)).astype(np.float32)
        u = r.normal(0, 1, (rows, width)).astype(np.float32)
        dg, du = dev(g), dev(u)
    e32, e16 = oracle.swiglu(np.ascontiguousarray(g), np.ascontiguousarray(u), want_bf16=True)
    h32, h16 = q.native_mlp_gate(dg, du, want_bf16=True, out_f32=nan_like((rows, width)))
    assert f32_close(h32, e32) and bf16_close(h16, e16, oracle)
    only16 = q.native_mlp_gate(dg, du, want_f32=False, want_bf16=True)[1]
    assert bf16_close(only16, e16, oracle)


def test_swiglu_edges(q, oracle):
    g = np.array([[0.0, -0.0, 1.0, -1.0, 30.0, -30.0, 100.0, -100.0, 88.0, -88.0, 1e-30, -1e-30]],
                 np.float32)
    u = np.full_like(g, 3.0)
    e32, _ = oracle.swiglu(g, u)
    h32, _ = q.native_mlp_gate(dev(g), dev(u))
    assert f32_close(h32, e32)
    assert np.array_equal(np.signbit(h32.cpu().numpy()), np.signbit(e32))


# ---------------------------------------------------------------- workspace

def test_workspace_arena(q):
    ctx = q.Context(0)
    ctx.ws_reserve(1 << 20)
    used, cap, _ = ctx.ws_stats()
    assert used == 0 and cap >= 1 << 20
    a = ctx.ws_tensor((100, 3))
    mark = ctx.ws_mark()
    b = ctx.ws_tensor((10,), torch.bfloat16)
    assert b.data_ptr() % 256 == 0 and b.data_ptr() >= a.data_ptr() + 1200
    ctx.ws_release(mark)
    c = ctx.ws_tensor((10,), torch.bfloat16)
    assert c.data_ptr() == b.data_ptr()  # slot reused by call order
    with pytest.raises(q.QdcError):
        ctx.ws_alloc(cap)  # exhausted -> QDC_ENOMEM, nothing allocated
    ctx.ws_reset()
    assert ctx.ws_tensor((1,)).data_ptr() == a.data_ptr()
    a.fill_(1.0)
    torch.cuda.synchronize()
    ctx.close()


@pytest.mark.parametrize("tokens,qh,kh,dim,rotary", [(33, 8, 2, 256, 64), (17, 4, 2, 64, 16),
                                                     (9, 2, 1, 4, 4), (1, 8, 2, 256, 64),
                                                     (65, 3, 1, 128, 128), (5, 2, 2, 96, 32)])
def test_q_k_norm_rope_one_launch(q, oracle, tokens, qh, kh, dim, rotary):
    """Query and key heads of the packed [q;gate | k | v] projection in one
    launch, each against the oracle."""
    r = rng(tokens + qh + dim)
    width = qh * 2 * dim + 2 * kh * dim
    proj = r.normal(0, 1, (tokens, width)).astype(np.float32)
    qgate = proj[:, :qh * 2 * dim].reshape(tokens, qh, 2 * dim)
    kraw = proj[:, qh * 2 * dim:qh * 2 * dim + kh * dim].reshape(tokens, kh, dim)
    wq = r.normal(0, 0.02, dim).astype(np.float32)
    wk = r.normal(0, 0.02, dim).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, rotary, 2048)
    eq = oracle.qk_norm_rope(np.ascontiguousarray(qgate[:, :, :dim]), wq, 1e-6, rotary, cos, sin,
                             seq_len=7)
    ek = oracle.qk_norm_rope(np.ascontiguousarray(kraw), wk, 1e-6, rotary, cos, sin, seq_len=7)
    dproj = dev(proj)
    dq = dproj[:, :qh * 2 * dim].view(tokens, qh, 2 * dim)[:, :, :dim]
    dk = dproj[:, qh * 2 * dim:qh * 2 * dim + kh * dim].view(tokens, kh, dim)
    dc, ds = q.rope_table(1e7, rotary, 2048, device="cuda")
    gq, gk = q.native_q_k_norm_rope(dq, dk, dev(wq), dev(wk), 1e-6, rotary, dc, ds, seq_len=7,
                                    q_out=nan_like((tokens, qh, dim)), k_out=nan_like((tokens, kh, dim)))
    assert f32_close(gq, eq) and f32_close(gk, ek)


def test_c_abi_rejects_bad_arguments_before_launch(q):
    """Host-only fault tests through the raw C ABI: NULL pointers, bad sizes,
    bad dtype, tables too short for the positions, aliasing -- each returns
    QDC_EINVAL with a message and launches nothing."""
    import ctypes
    lib = q.load()
    ctx = q.context(0)
    h = ctx.handle
    x = torch.zeros((4, 8), device="cuda")
    y = torch.zeros((4, 8), device="cuda")
    p = ctypes.c_void_p(x.data_ptr())
    p2 = ctypes.c_void_p(y.data_ptr())
    g = ctypes.c_void_p(torch.zeros(8, device="cuda").data_ptr())
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    EINVAL = 1
    cases = [
        lambda: lib.qdc_residual_rms(h, None, p2, None, None, g, 1e-6, 1, 4, 8, 8, 8, 8, 8, 0, s),  # x NULL
        lambda: lib.qdc_residual_rms(h, None, p, p, None, g, 1e-6, 1, 4, 8, 8, 8, 8, 8, 0, s),  # y aliases x
        lambda: lib.qdc_residual_rms(h, None, p2, p, None, g, 1e-6, 1, 4, 8, 4, 8, 8, 8, 0, s),  # ld < width
        lambda: lib.qdc_residual_rms(h, None, p2, p, None, g, 1e-6, 1, 4, 8, 8, 8, 8, 8, 7, s),  # dtype
        lambda: lib.qdc_residual_rms(h, None, p2, p, None, g, 1e-6, 1, -1, 8, 8, 8, 8, 8, 0, s),  # rows
        lambda: lib.qdc_residual_rms(h, None, p2, p, None, None, 1e-6, 1, 4, 8, 8, 8, 8, 8, 0, s),  # gamma
        lambda: lib.qdc_swiglu(h, None, None, p, p, 4, 8, 8, 8, 8, s),
        lambda: lib.qdc_swiglu(h, p, None, None, p, 4, 8, 8, 8, 8, s),
        lambda: lib.qdc_gated_rms(h, p, p, None, 4, 2, 4, 8, 8, 0, 8, g, 1e-6, s),
        lambda: lib.qdc_gated_rms(h, p, p, p, 4, 2, 4, 8, 4, 0, 8, g, 1e-6, s),
        lambda: lib.qdc_qk_norm_rope(h, p, p, 4, 2, 4, 8, 4, g, 1e-6, 3, p, p, 4, 0, 0, s),
        lambda: lib.qdc_qk_norm_rope(h, p, p, 4, 2, 4, 8, 4, g, 1e-6, 4, p, p, 2, 0, 0, s),
        lambda: lib.qdc_qk_norm_rope(h, p, p, 4, 2, 4, 8, 4, g, 1e-6, 4, None, None, 8, 0, 0, s),
        lambda: lib.qdc_q_k_norm_rope(h, p, p, p, p, 4, 2, 0, 4, 8, 4, 8, 4, g, g, 1e-6, 0, None, None,
                                      0, 0, 0, s),
        lambda: lib.qdc_gather_rms_device_ids(h, p, None, None, p, None, None, 1e-6, 1, 4, 8, 64, 0, s),
        lambda: lib.qdc_gather_rms_device_ids(h, None, None, p, p, None, None, 1e-6, 1, 4, 8, 64, 0, s),
        lambda: lib.qdc_ws_alloc(h, 16, 100, ctypes.byref(ctypes.c_void_p())),
        lambda: lib.qdc_ws_release(h, 1 << 40),
    ]
    for i, call in enumerate(cases):
        assert call() == EINVAL, i
        assert lib.qdc_last_error(h), i
    torch.cuda.synchronize()
    assert torch.count_nonzero(x).item() == 0 and torch.count_nonzero(y).item() == 0  # nothing ran


# ------------------------------------------------------- DeltaNet prologue

@pytest.mark.parametrize("tokens,seq_len,kh,kd,vh,vd,pad", [
    (200, 64, 2, 128, 4, 128, 8),      # config 1 shape, vector path
    (130, 0, 16, 128, 16, 128, 16),    # config 5 heads, one sequence, tail run
    (37, 10, 2, 128, 2, 128, 0),       # sequences shorter than a run
    (9, 3, 1, 2, 2, 2, 7),             # fixture dims, generic path
    (50, 25, 2, 64, 3, 96, 4),         # generic head widths
    (1, 0, 2, 128, 4, 128, 8),
    (48, 7, 2, 128, 4, 128, 0),        # exactly one pipeline tile, short sequences
    (49, 0, 16, 128, 16, 128, 0),      # one token past a tile
    (4100, 2048, 4, 128, 8, 128, 32),  # sequence starts inside tiles (2048 = 42 x 48 + 32)
])
def test_delta_conv_norm(q, oracle, tokens, seq_len, kh, kd, vh, vd, pad):
    r = rng(tokens + kd + vd)
    C = 2 * kh * kd + vh * vd
    proj = r.normal(0, 1, (tokens, C + pad)).astype(np.float32)
    w = r.normal(0, 0.5, (C, 1, 4)).astype(np.float32)
    eq, ek, ev = oracle.delta_conv_norm(proj, w.reshape(C, 4), kh, kd, vh, vd, seq_len=seq_len or None)
    gq, gk, gv = q.native_delta_conv_norm(dev(proj), dev(w), kh, kd, vh, vd, seq_len=seq_len or None,
                                          q_out=nan_like((tokens, kh, kd)), k_out=nan_like((tokens, kh, kd)),
                                          v_out=nan_like((tokens, vh, vd)))
    assert f32_close(gq, eq) and f32_close(gk, ek) and f32_close(gv, ev)


@pytest.mark.parametrize("B,S,H,D", [(2, 33, 8, 256), (1, 64, 4, 64), (3, 5, 2, 4), (2, 17, 3, 128)])
def test_attn_gate(q, oracle, B, S, H, D):
    """values * sigmoid(gate) from an attention output in (B, H, S, D) and
    the gate half of the packed [q;gate] projection."""
    r = rng(B * S + H * D)
    values = r.normal(0, 1, (B, S, H, D)).astype(np.float32)   # stored (B, S, H, D), viewed (B, H, S, D)
    proj = r.normal(0, 2, (B * S, H, 2 * D)).astype(np.float32)
    vt = values.transpose(0, 2, 1, 3)
    expected = oracle.attn_gate(np.ascontiguousarray(vt), np.ascontiguousarray(proj[:, :, D:]))
    dv = dev(values).transpose(1, 2)
    dp = dev(proj)
    got = q.native_attn_gate(dv, dp[:, :, D:], out=nan_like((B * S, H * D)))
    assert f32_close(got, expected)


@pytest.mark.parametrize("tokens,heads,lead,tail", [(4096, 16, 6144 + 2048, 0), (33, 4, 9, 3),
                                                    (1, 1, 0, 0), (0, 8, 5, 0), (257, 48, 17, 1)])
def test_delta_gates(q, oracle, tokens, heads, lead, tail):
    """beta / decay from the a, b columns at the tail of packed projection
    rows (src/backbone.jl:292-297), including |a + dt_bias| up to ~60."""
    r = rng(tokens + heads)
    proj = r.normal(0, 20, (tokens, lead + 2 * heads + tail)).astype(np.float32)
    a_decay = -np.exp(r.normal(0, 1, heads)).astype(np.float32)
    dt_bias = r.normal(0, 1, heads).astype(np.float32)
    eb, ed = oracle.delta_gates(proj, lead, heads, a_decay, dt_bias)
    gb, gd = q.native_delta_gates(dev(proj), lead, heads, dev(a_decay), dev(dt_bias),
                                  beta=nan_like((tokens, heads)), decay=nan_like((tokens, heads)))
    assert f32_close(gb, eb) and f32_close(gd, ed)


def test_delta_gates_rejects_bad_columns(q):
    proj = torch.zeros((4, 10), device="cuda")
    h = torch.zeros(4, device="cuda")
    with pytest.raises(q.DimensionMismatch):
        q.native_delta_gates(proj, 3, 4, h, h)   # 3 + 8 > 10
    with pytest.raises(q.DimensionMismatch):
        q.native_delta_gates(proj, 0, 4, h[:3], h)


@pytest.mark.parametrize("width_heads", [16, 8])
def test_row_kernel_waits_for_its_producer(q, oracle, width_heads):
    """With programmatic dependent launch on, a residual norm issued right
    behind the gated norm that writes its input (a NaN-filled buffer) must
    read the finished rows, never the fill."""
    T, H, D = 16384, width_heads, 128
    r = rng(T + H)
    o = r.normal(0, 1, (T, H, D)).astype(np.float32)
    z = r.normal(0, 1, (T, H, D)).astype(np.float32)
    wg = (1 + r.normal(0, 0.02, D)).astype(np.float32)
    m = r.normal(0, 1, (T, H * D)).astype(np.float32)
    wr = r.normal(0, 0.02, H * D).astype(np.float32)
    gated = oracle.gated_rms(o, z, wg, 1e-6)
    ex_r, ex_y = oracle.residual_rms(gated, m, wr, 1e-6)
    do, dz, dwg, dm, dwr = dev(o), dev(z), dev(wg), dev(m), dev(wr)
    ctx = q.context(torch.device("cuda", 0))
    before = ctx.pdl
    try:
        ctx.pdl = True  # QDC_OPT_PDL (the default): the launch mode in which the wait matters
        for _ in range(3):
            g = nan_like((T, H * D))
            q.native_gated_rms(do, dz, dwg, 1e-6, out=g, ctx=ctx)
            rr, yy = q.native_residual_rms(g, dm, dwr, 1e-6, out_r=nan_like((T, H * D)),
                                           out_y=nan_like((T, H * D)), ctx=ctx)
            assert not torch.isnan(yy).any()
            assert f32_close(rr, ex_r) and f32_close(yy, ex_y)
    finally:
        ctx.pdl = before


def _misaligned(a):
    """A device copy of float32 `a` that starts 4 bytes past a 16-byte
    boundary (the vector kernels read gamma as float4; the host must route
    such a gamma to the scalar kernels)."""
    a = np.ascontiguousarray(a, np.float32)
    buf = torch.empty(a.size + 4, dtype=torch.float32, device="cuda")
    view = buf[1:1 + a.size]
    view.copy_(torch.from_numpy(a))
    assert view.data_ptr() % 16 == 4
    return view


def test_misaligned_gamma_takes_scalar_kernels(q, oracle):
    r = rng(5)
    x = r.normal(0, 1, (37, 1024)).astype(np.float32)
    m = r.normal(0, 1, (37, 1024)).astype(np.float32)
    w = r.normal(0, 0.02, 1024).astype(np.float32)
    er, ey = oracle.residual_rms(x, m, w, 1e-6)
    rr, yy = q.native_residual_rms(dev(x), dev(m), _misaligned(w), 1e-6)
    assert f32_close(rr, er) and f32_close(yy, ey)
    table = r.normal(0, 0.02, (500, 1024)).astype(np.float32)
    ids = r.integers(0, 500, 37).astype(np.int32)
    ex, ey = oracle.gather_rms(table, ids, m, w, 1e-6)
    gx, gy = q.native_gather_rms(dev(table), ids, _misaligned(w), 1e-6, add=dev(m))
    assert np.array_equal(gx.cpu().numpy(), ex) and f32_close(gy, ey)
    o = r.normal(0, 1, (37, 4, 128)).astype(np.float32)
    z = r.normal(0, 1, (37, 4, 128)).astype(np.float32)
    wg = (1 + r.normal(0, 0.02, 128)).astype(np.float32)
    assert f32_close(q.native_gated_rms(dev(o), dev(z), _misaligned(wg), 1e-6),
                     oracle.gated_rms(o, z, wg, 1e-6))
    qi = r.normal(0, 1, (37, 8, 256)).astype(np.float32)
    ki = r.normal(0, 1, (37, 2, 256)).astype(np.float32)
    wq = r.normal(0, 0.02, 256).astype(np.float32)
    wk = r.normal(0, 0.02, 256).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, 64, 37)
    dc, ds = q.rope_table(1e7, 64, 37, device="cuda")
    gq, gk = q.native_q_k_norm_rope(dev(qi), dev(ki), _misaligned(wq), dev(wk), 1e-6, 64, dc, ds)
    assert f32_close(gq, oracle.qk_norm_rope(qi, wq, 1e-6, 64, cos, sin))
    assert f32_close(gk, oracle.qk_norm_rope(ki, wk, 1e-6, 64, cos, sin))


# ----------------------------------------------------------- bf16 storage

@pytest.mark.parametrize("offset", [0, 1, 3])
def test_bf16_widen_every_pattern(q, offset):
    """qdc_bf16_to_f32 = bits << 16 (src/safetensors.jl:28-30) for all 65,536
    patterns (NaN payloads included), aligned and misaligned, odd lengths."""
    bits = np.arange(65536 + 5, dtype=np.uint32).astype(np.uint16)
    buf = torch.from_numpy(np.concatenate([np.zeros(offset, np.uint16), bits]).view(np.int16)).cuda()
    src = buf[offset:]
    got = q.native_bf16_to_f32(src)
    expected = (bits.astype(np.uint32) << 16)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), expected)
    out = torch.zeros(7, device="cuda")
    q.native_bf16_to_f32(src[:7], out=out)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), expected[:7])
    assert q.native_bf16_to_f32(src[:0]).numel() == 0


@pytest.mark.parametrize("offset", [0, 1])
def test_bf16_encode_matches_reference_rounding(q, oracle, offset):
    """qdc_f32_to_bf16: round to nearest even by integer add, no NaN special
    case (src/safetensors.jl:38-42), bit-exact with the oracle."""
    r = rng(9)
    x = np.concatenate([r.normal(0, 1, 40001).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8,
                                  3.4028235e38, 1e-40, -1e-40], np.float32),
                        (np.arange(4096, dtype=np.uint32) * 0x00010001 + 0x7fff).view(np.float32)])
    buf = torch.from_numpy(np.concatenate([np.zeros(offset, np.float32), x])).cuda()
    got = q.native_f32_to_bf16(buf[offset:])
    assert got.dtype == torch.bfloat16
    assert np.array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16), oracle.bf16_encode(x))


def test_bf16_converters_reject_overlap_and_bad_types(q):
    t = torch.zeros(64, device="cuda")
    with pytest.raises(q.ArgumentError):
        q.native_bf16_to_f32(t)                      # Float32 is not bf16 bits
    with pytest.raises(q.ArgumentError):
        q.native_f32_to_bf16(t.view(torch.int32))    # not Float32
    with pytest.raises(q.ArgumentError):             # out overlaps in
        q.native_f32_to_bf16(t, out=t.view(torch.bfloat16)[:64])


def _write_bf16_checkpoint(src_dir, dst_dir, oracle):
    """The fixture checkpoint with every tensor stored as BF16."""
    import json
    import shutil
    import struct
    from qdc_b200.model import read_safetensors
    shutil.copyfile(os.path.join(src_dir, "config.json"), os.path.join(dst_dir, "config.json"))
    tensors = read_safetensors(os.path.join(src_dir, "model.safetensors"))
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        bits = oracle.bf16_encode(np.ascontiguousarray(arr, np.float32).reshape(-1)).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(arr.shape), "data_offsets": [off, off + len(bits)]}
        blobs.append(bits)
        off += len(bits)
    h = json.dumps(header).encode()
    with open(os.path.join(dst_dir, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def test_bf16_checkpoint_upload_matches_host_widening(q, oracle, tmp_path):
    """from_directory uploads BF16 tensors as raw bits and widens them on the
    device; the model equals one built from host-widened weights."""
    from qdc_b200.model import load_weights
    _write_bf16_checkpoint(GOLDEN, str(tmp_path), oracle)
    dev_model = q.QwenBackbone.from_directory(str(tmp_path), device="cuda")
    cfg, host_w = load_weights(str(tmp_path))           # widened on the host
    _, raw_w = load_weights(str(tmp_path), raw_bf16=True)
    assert raw_w["embed_tokens.weight"].dtype == np.uint16
    host_model = q.QwenBackbone(cfg, host_w, device="cuda")
    assert torch.equal(dev_model.embedding, host_model.embedding)
    for a, b in zip(dev_model.layers, host_model.layers):
        for k in a:
            if torch.is_tensor(a[k]):
                assert torch.equal(a[k], b[k]), k
    ids = (np.arange(33) * 5) % 64
    mask = np.ones(33, np.int64)
    assert np.array_equal(q.backbone_hidden(dev_model, ids, mask), q.backbone_hidden(host_model, ids, mask))


def test_pdl_option(q, oracle):
    """QDC_OPT_PDL (on by default) launches the same kernels with
    programmatic dependent launch: identical results with it off and on; an
    unknown option is refused."""
    from qdc_b200 import _lib
    ctx = q.context(torch.device("cuda", 0))
    assert ctx.pdl
    r = rng(3)
    x = r.normal(0, 1, (300, 1024)).astype(np.float32)
    m = r.normal(0, 1, (300, 1024)).astype(np.float32)
    w = r.normal(0, 0.02, 1024).astype(np.float32)
    try:
        ctx.pdl = False
        off = q.native_residual_rms(dev(x), dev(m), dev(w), 1e-6, ctx=ctx)
        ref = q.native_residual_rms(off[1], dev(m), dev(w), 1e-6, ctx=ctx)
    finally:
        ctx.pdl = True
    g = nan_like((300, 1024))
    q.native_residual_rms(dev(x), dev(m), dev(w), 1e-6, out_y=g, ctx=ctx)  # producer ...
    on = q.native_residual_rms(g, dev(m), dev(w), 1e-6, ctx=ctx)       # ... and consumer
    assert torch.equal(on[0], ref[0]) and torch.equal(on[1], ref[1])
    with pytest.raises(q.ArgumentError):
        _lib.check(ctx.lib.qdc_set_option(ctx.handle, 99, 1), ctx.handle)


@pytest.mark.parametrize("kd,vd", [(128, 128), (8, 6)])
def test_delta_conv_norm_edge_values(q, oracle, kd, vd):
    """The fused L2 norm on the reference's edge values (test/backbone.jl:
    290-313): 0, -0, NaN, Inf, floatmax, the smallest subnormal, each token
    its own sequence and a conv that passes the current token through, so
    every head of token t holds silu(edge[t])."""
    edges = np.array([0.0, -0.0, np.nan, np.inf, np.finfo(np.float32).max, 1e-45], np.float32)
    kh, vh = 2, 4
    C = 2 * kh * kd + vh * vd
    proj = np.repeat(edges[:, None], C + 4, axis=1).astype(np.float32)
    w = np.zeros((C, 4), np.float32)
    w[:, 3] = 1.0  # taps oldest first: tap 3 is the current token
    eq, ek, ev = oracle.delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len=1)
    gq, gk, gv = q.native_delta_conv_norm(dev(proj), dev(w), kh, kd, vh, vd, seq_len=1,
                                          q_out=nan_like((6, kh, kd)), k_out=nan_like((6, kh, kd)),
                                          v_out=nan_like((6, vh, vd)))
    for got, exp in ((gq, eq), (gk, ek), (gv, ev)):
        assert f32_close(got, exp)
        a = got.cpu().numpy()
        assert np.array_equal(np.isnan(a), np.isnan(exp)) and np.array_equal(np.isinf(a), np.isinf(exp))


def test_plain_gather_entry_point(q, oracle):
    """qdc_gather (the boundary's plain gather): bit-exact rows, host ids
    checked before launch."""
    import ctypes
    from qdc_b200 import _lib, ops
    ctx = q.context(torch.device("cuda", 0))
    r = rng(21)
    V, H, n = 1000, 1024, 77
    table = r.normal(0, 0.02, (V, H)).astype(np.float32)
    ids = r.integers(0, V, n).astype(np.int32)
    out = nan_like((n, H))
    dt = dev(table)
    st = ctx.lib.qdc_gather(ctx.handle, ops._ptr(out), ops._ptr(dt), ids.ctypes.data_as(ctypes.c_void_p),
                            n, H, V, _lib.QDC_F32, ops._stream(torch.device("cuda", 0)))
    _lib.check(st, ctx.handle)
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), table[ids])
    bad = ids.copy()
    bad[5] = V
    st = ctx.lib.qdc_gather(ctx.handle, ops._ptr(out), ops._ptr(dt), bad.ctypes.data_as(ctypes.c_void_p),
                            n, H, V, _lib.QDC_F32, ops._stream(torch.device("cuda", 0)))
    assert st == _lib.QDC_EBOUNDS


def test_delta_conv_norm_negative_zero_window(q, oracle):
    """All taps -0 inside one long sequence (the pipeline's branch-free path):
    the conv starts from +0 as the reference's `value = 0; value += x * w`
    does, so every output is +0, sign included."""
    kh, kd, vh, vd, tokens = 2, 128, 4, 128, 200
    C = 2 * kh * kd + vh * vd
    proj = np.full((tokens, C), -0.0, np.float32)
    w = rng(4).normal(0, 0.5, (C, 4)).astype(np.float32)
    eq, ek, ev = oracle.delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len=None)
    gq, gk, gv = q.native_delta_conv_norm(dev(proj), dev(w), kh, kd, vh, vd)
    for got, exp in ((gq, eq), (gk, ek), (gv, ev)):
        a = got.cpu().numpy()
        assert np.array_equal(a, exp) and np.array_equal(np.signbit(a), np.signbit(exp))
        assert not np.signbit(exp).any()


@pytest.mark.parametrize("batch,n,width,ld_pad", [(300, 64, 256, 0), (7, 64, 128, 64), (5, 17, 100, 3),
                                                  (3, 1, 5, 0), (2, 64, 1, 0), (1, 33, 300, 0)])
def test_delta_solve(q, oracle, batch, n, width, ld_pad):
    """delta_solve in place (UnitLowerTriangular(system) \\ rhs,
    src/backbone.jl:279) against the oracle's forward substitution, with
    the right-hand side a column slice of a wider buffer (as the chunked
    delta rule solves [V*beta | K*beta*exp(cum)] in one go) and garbage on
    and above the diagonal of system, which must not be read.  Entries
    of system in [-0.3, 0.3] (the delta rule's are beta * k_i.k_j * decay,
    at most 1 in magnitude)."""
    rng = np.random.default_rng(batch * n + width)
    system = rng.uniform(-0.3, 0.3, (batch, n, n)).astype(np.float32)
    system += np.triu(np.full((n, n), 7.0, np.float32))
    rhs = rng.standard_normal((batch, n, width + ld_pad), dtype=np.float32)
    expected = oracle.unit_lower_solve(system, np.ascontiguousarray(rhs[:, :, :width]))
    dsys = torch.from_numpy(system).cuda()
    drhs = torch.from_numpy(rhs).cuda()
    got = q.native_delta_solve(dsys, drhs[:, :, :width])
    scale = np.abs(expected).max(axis=1, keepdims=True) + 1e-30
    a = got.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(a - expected) <= 1e-5 * scale + 1e-6)
    assert np.array_equal(drhs[:, :, width:].cpu().numpy(), rhs[:, :, width:])  # pad untouched
    assert np.array_equal(dsys.cpu().numpy(), system)


def test_delta_solve_rejects_bad_arguments(q):
    x = torch.zeros((2, 65, 8), device="cuda")
    with pytest.raises(q.ArgumentError):
        q.native_delta_solve(torch.zeros((2, 65, 65), device="cuda"), x)
    with pytest.raises(q.DimensionMismatch):
        q.native_delta_solve(torch.zeros((2, 4, 4), device="cuda"), torch.zeros((2, 5, 8), device="cuda"))


@pytest.mark.parametrize("tokens,seq_len", [(77, None), (300, 128)])
def test_qk_norm_rope_head_major_output(q, oracle, tokens, seq_len):
    """Output by strides (qdc_qk_norm_rope_strided): q written head-major,
    the (dim, tokens, heads) Julia array the reference's attention GEMMs
    read (ext/cuda_attention.jl:125-154), and K expanded to every query
    head by one call per group (query head h reads kv head h // groups), as
    prepare_head_kernel! lays it out; plus an output whose head stride is
    not a multiple of 4 (the scalar kernel).  Against the oracle."""
    r = rng(tokens)
    Hq, Hkv, D, R = 8, 2, 256, 64
    G = Hq // Hkv
    proj = r.normal(0, 1, (tokens, Hq * 2 * D + Hkv * D)).astype(np.float32)
    gq = r.normal(0, 0.02, D).astype(np.float32)
    gk = r.normal(0, 0.02, D).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, R, 512)
    qg = proj[:, :Hq * 2 * D].reshape(tokens, Hq, 2 * D)
    kr = proj[:, Hq * 2 * D:].reshape(tokens, Hkv, D)
    eq = oracle.qk_norm_rope(np.ascontiguousarray(qg[:, :, :D]), gq, 1e-6, R, cos, sin, seq_len=seq_len)
    ek = oracle.qk_norm_rope(np.ascontiguousarray(kr), gk, 1e-6, R, cos, sin, seq_len=seq_len)
    dp, dc, ds = dev(proj), dev(cos), dev(sin)
    dq = dp[:, :Hq * 2 * D].view(tokens, Hq, 2 * D)[:, :, :D]
    dk = dp[:, Hq * 2 * D:].view(tokens, Hkv, D)
    q_hm = nan_like((Hq, tokens, D))
    q.native_qk_norm_rope(dq, dev(gq), 1e-6, R, dc, ds, seq_len=seq_len, out=q_hm.permute(1, 0, 2))
    assert f32_close(q_hm.permute(1, 0, 2), eq)
    k_exp = nan_like((Hq, tokens, D))
    for g in range(G):
        q.native_qk_norm_rope(dk, dev(gk), 1e-6, R, dc, ds, seq_len=seq_len, out=k_exp[g::G].permute(1, 0, 2))
    for h in range(Hq):
        assert f32_close(k_exp[h], ek[:, h // G])
    padded = nan_like((tokens, Hq, D + 1))
    q.native_qk_norm_rope(dq, dev(gq), 1e-6, R, dc, ds, seq_len=seq_len, out=padded[:, :, :D])
    assert f32_close(padded[:, :, :D], eq)
    assert torch.isnan(padded[:, :, D]).all()


@pytest.mark.parametrize("tokens,seq_len,kh,kd,vh,vd", [(300, 128, 2, 128, 4, 128), (130, 0, 1, 128, 3, 128),
                                                        (50, 25, 2, 64, 3, 96)])
def test_delta_conv_norm_v_into_mixed_rows(q, oracle, tokens, seq_len, kh, kd, vh, vd):
    """v written through a token stride (qdc_delta_conv_norm_strided) into the
    value rows of a (tokens, qkv width) buffer -- the conv output `mixed`
    the reference's delta-rule kernels read v from (ext/cuda_delta.jl:199) --
    on the pipeline, register and scalar kernels; the other rows untouched."""
    r = rng(tokens + vh)
    C = 2 * kh * kd + vh * vd
    proj = r.normal(0, 1, (tokens, C + 4)).astype(np.float32)
    w = r.normal(0, 0.5, (C, 4)).astype(np.float32)
    eq, ek, ev = oracle.delta_conv_norm(proj, w, kh, kd, vh, vd, seq_len=seq_len or None)
    mixed = nan_like((tokens, C))
    v_view = mixed[:, 2 * kh * kd:].view(tokens, vh, vd)
    gq, gk, gv = q.native_delta_conv_norm(dev(proj), dev(w), kh, kd, vh, vd, seq_len=seq_len or None,
                                          v_out=v_view)
    assert f32_close(gq, eq) and f32_close(gk, ek) and f32_close(v_view, ev)
    assert torch.isnan(mixed[:, :2 * kh * kd]).all()
