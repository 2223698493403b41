"""Host-side logic of qdc_b200.QwenBackbone on the CPU: weight loading and
packing, the torch stand-ins for the out-of-scope parts (causal attention
with the reference's -floatmax mask, 4-tap causal conv, chunked gated delta
rule), the layer orchestration and input validation.

The per-layer kernels need a B200, so for this CPU test ONLY they are
replaced, through monkeypatch, by test doubles built on the oracle; the
product itself has no CPU path (QwenBackbone refuses a non-CUDA device).
The GPU suite (test_gpu_backbone.py) runs the same forward on the real
kernels."""
import threading

import numpy as np
import pytest
import torch

from conftest import GOLDEN


class _Ctx:
    lock = threading.RLock()

    def sync(self, stream=None):
        pass


class _HostWorkspace:
    """CPU stand-in for the model's workspace arena (test double): the same
    begin / take / mark / release in carve order, with the arena's 256-byte
    alignment, over one CPU byte buffer.  It records the high-water mark of
    each forward so the tests can check the forward stays inside the bytes
    forward_bytes planned for it."""

    def __init__(self):
        self.buf = None
        self.cursor = self.high = self.planned = 0
        self.generation = 0
        self.takes = []

    def begin(self, nbytes):
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(int(nbytes), dtype=torch.uint8)
            self.generation += 1
        self.cursor, self.planned, self.high = 0, int(nbytes), 0
        self.takes = []

    def take(self, shape, dtype=torch.float32):
        n = int(np.prod(shape)) * torch.empty((), dtype=dtype).element_size()
        start = (self.cursor + 255) // 256 * 256
        assert start + max(n, 1) <= self.planned, "forward carved more than forward_bytes planned"
        self.cursor = start + max(n, 1)
        self.high = max(self.high, self.cursor)
        self.takes.append((start, tuple(shape), dtype))
        return self.buf[start:start + n].view(dtype).view(tuple(int(d) for d in shape))

    def take_all(self, spec):
        return {name: self.take(shape, dtype) for name, (shape, dtype) in spec.items()}

    def mark(self):
        return self.cursor

    def release(self, mark):
        self.cursor = mark


def _put(out, arr):
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if out is None:
        return t
    out.copy_(t.view(out.shape))
    return out


@pytest.fixture
def cpu_backbone(monkeypatch, oracle):
    from qdc_b200 import backbone as BB
    from qdc_b200 import ops
    from qdc_b200.model import pack_layers

    n = lambda t: t.detach().cpu().numpy()
    c = lambda a: np.ascontiguousarray(a)

    def gather_rms(emb, ids, w, eps, ctx=None, out_x=None, out_y=None, **k):
        r, y = oracle.gather_rms(n(emb), np.asarray(ids, np.int32), None, n(w), eps)
        return _put(out_x, r), _put(out_y, y)

    def residual_rms(x, m, w, eps, ctx=None, out_r=None, out_y=None, store_residual=True, **k):
        r, y = oracle.residual_rms(c(n(x)), c(n(m)), n(w), eps)
        return (_put(out_r, r) if store_residual else None), _put(out_y, y)

    def residual_add_rms(r, m, w, eps, ctx=None, out_y=None, **k):
        rr, y = oracle.residual_rms(c(n(r)), c(n(m)), n(w), eps)
        _put(r, rr)
        return r, _put(out_y, y)

    def qk(x, w, eps, rot, cos, sin, pos_offset=0, seq_len=None, ctx=None, out=None, **k):
        return _put(out, oracle.qk_norm_rope(c(n(x)), n(w), eps, rot, n(cos), n(sin), pos_offset=pos_offset,
                                             seq_len=seq_len))

    def q_k(qi, ki, wq, wk, eps, rot, cos, sin, seq_len=None, ctx=None, q_out=None, k_out=None, **k):
        return (_put(q_out, oracle.qk_norm_rope(c(n(qi)), n(wq), eps, rot, n(cos), n(sin), seq_len=seq_len)),
                _put(k_out, oracle.qk_norm_rope(c(n(ki)), n(wk), eps, rot, n(cos), n(sin), seq_len=seq_len)))

    def gated(o, z, w, eps, ctx=None, out=None, **k):
        # the kernel's layout contract: heads contiguous within a token
        assert o.stride(1) == o.shape[2] and z.stride(1) == z.shape[2]
        return _put(out, oracle.gated_rms(c(n(o)), c(n(z)), n(w), eps))

    def swiglu(g, u, ctx=None, out_f32=None, **k):
        return _put(out_f32, oracle.swiglu(c(n(g)), c(n(u)))[0]), None

    def conv_norm(proj, w, kh, kd, vh, vd, seq_len=None, ctx=None, q_out=None, k_out=None, v_out=None, **k):
        C = 2 * kh * kd + vh * vd
        q, kk, v = oracle.delta_conv_norm(c(n(proj))[:, :C], n(w).reshape(C, 4), kh, kd, vh, vd,
                                          seq_len=seq_len)
        return _put(q_out, q), _put(k_out, kk), _put(v_out, v)

    def delta_gates(proj, start, heads, a_decay, dt_bias, ctx=None, beta=None, decay=None, **k):
        b, d = oracle.delta_gates(c(n(proj)), start, heads, n(a_decay), n(dt_bias))
        return _put(beta, b), _put(decay, d)

    def attn_gate(values, gate, ctx=None, out=None, **k):
        return _put(out, oracle.attn_gate(c(n(values)), c(n(gate))))

    def delta_solve(system, x, ctx=None, **k):
        return _put(x, oracle.unit_lower_solve(n(system), n(x)))

    def rope_table(theta, r, rows, device=None):
        cs, sn = oracle.rope_table(theta, r, rows)
        return torch.from_numpy(cs), torch.from_numpy(sn)

    for name, fn in (("native_gather_rms", gather_rms), ("native_residual_rms", residual_rms),
                     ("native_residual_add_rms", residual_add_rms), ("native_q_k_norm_rope", q_k),
                     ("native_qk_norm_rope", qk),
                     ("native_gated_rms", gated), ("native_mlp_gate", swiglu),
                     ("native_delta_conv_norm", conv_norm), ("native_delta_gates", delta_gates),
                     ("native_attn_gate", attn_gate), ("native_delta_solve", delta_solve),
                     ("rope_table", rope_table)):
        monkeypatch.setattr(ops, name, fn)

    def make(config, weights):
        b = BB.QwenBackbone.__new__(BB.QwenBackbone)
        b.config, b.device, b.ctx, b.ws = config, torch.device("cpu"), _Ctx(), _HostWorkspace()
        b.embedding = BB._device_f32(weights["embed_tokens.weight"], "cpu")
        b.final_norm = BB._device_f32(weights["norm.weight"], "cpu")
        b.layers = pack_layers(config, weights, "cpu")
        b._init_caches()
        return b

    return make


def test_product_refuses_cpu_device():
    import qdc_b200
    from qdc_b200.model import load_weights
    cfg, w = load_weights(GOLDEN)
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.QwenBackbone(cfg, w, device="cpu")


@pytest.mark.parametrize("n,holes", [(1, False), (9, True), (64, False), (65, True), (129, True)])
def test_fixture_forward_orchestration(cpu_backbone, n, holes):
    import qdc_b200
    from oracle import forward as F
    from qdc_b200.model import load_weights
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    ids = np.arange(n) % 64
    mask = np.ones(n, np.int64)
    if holes and n > 1:
        mask[0:n - 1:3] = 0
    actual = qdc_b200.backbone_hidden(model, ids, mask)
    expected = F.backbone_hidden(F.load_model(GOLDEN), ids, mask)
    assert np.all(np.abs(actual - expected) <= 2e-5 + 2e-5 * np.abs(expected))
    assert np.array_equal(qdc_b200.backbone_hidden(model, ids, mask, positions=[1, n]),
                          actual[[0, n - 1]])


@pytest.mark.parametrize("n,holes", [(1, False), (9, True), (65, False), (66, True)])
def test_last_token_forward_orchestration(cpu_backbone, n, holes):
    """The last-token forward (one-query final attention, one-token final
    MLP) equals the last row of the all-token forward."""
    import qdc_b200
    from qdc_b200.model import load_weights
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    ids = (np.arange(n) * 7) % 64
    mask = np.ones(n, np.int64)
    if holes and n > 1:
        mask[0:n - 1:3] = 0
    full = qdc_b200.backbone_hidden(model, ids, mask)[-1]
    last = model.batch_hidden(ids.reshape(1, -1), mask.reshape(1, -1), last_only=True).numpy()[0]
    assert np.all(np.abs(last - full) <= 2e-5 + 2e-5 * np.abs(full))
    assert model.ws.high <= model.ws.planned


@pytest.mark.parametrize("scan", [True, False])
def test_chunked_delta_matches_token_recurrence(oracle, scan):
    """The chunked rule (zero-padded tail chunk), with the hand-off as a
    linear scan and per chunk, every intermediate in its own slot and the
    unit-lower-triangular solve by the oracle's forward substitution,
    equals the token recurrence of src/backbone_cpu.jl:681-705 on odd
    lengths."""
    from qdc_b200.backbone import _chunked_spec, chunked_delta
    g = torch.Generator().manual_seed(0)
    upper = torch.ones((64, 64), dtype=torch.bool).triu_(1)

    def solve(system, x):
        x.copy_(torch.from_numpy(oracle.unit_lower_solve(system.numpy(), x.numpy())))

    for S in (1, 63, 64, 65, 130):
        B, Hk, Dk, Hv, Dv = 2, 2, 8, 4, 6
        q = torch.nn.functional.normalize(torch.randn(B, S, Hk, Dk, generator=g), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(B, S, Hk, Dk, generator=g), dim=-1)
        v = torch.randn(B, S, Hv, Dv, generator=g)
        beta = torch.rand(B, S, Hv, generator=g)
        decay = -torch.rand(B, S, Hv, generator=g)
        slots = {name: torch.full(shape, float("nan")).to(dt)
                 for name, (shape, dt) in _chunked_spec(B, S, Hv, Dk, Dv, scan).items()}
        out = torch.full((B, S, Hv, Dv), float("nan"))
        assert chunked_delta(q, k, v, beta, decay, Hv // Hk, slots, out, upper, solve) is out
        out = out.double()
        for b in range(B):
            for h in range(Hv):
                kh = h // (Hv // Hk)
                state = torch.zeros(Dv, Dk, dtype=torch.float64)
                for t in range(S):
                    f = torch.exp(decay[b, t, h].double())
                    kt, qt = k[b, t, kh].double(), q[b, t, kh].double()
                    proj = beta[b, t, h].double() * (v[b, t, h].double() - f * (state @ kt))
                    state = f * state + torch.outer(proj, kt)
                    assert torch.allclose(out[b, t, h], state @ qt, atol=2e-5, rtol=2e-5)


def test_validation_before_any_work(cpu_backbone):
    import qdc_b200
    from qdc_b200.model import load_weights
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    for ids, mask in (([1, 2], [1]), ([], []), ([1, 2], [1, 2]), ([64], [1]), ([-1], [1])):
        with pytest.raises(qdc_b200.ArgumentError):
            qdc_b200.backbone_hidden(model, ids, mask)
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.backbone_hidden(model, [[1, 2], [3, 4]], [[1, 1], [1, 1]])
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.backbone_hidden(model, [1, 2, 3], [1, 1, 1], positions=[4])


def test_config_validation():
    from qdc_b200.model import Config
    import json
    import os
    with open(os.path.join(GOLDEN, "config.json")) as f:
        src = json.load(f)
    assert Config.from_json(src).rotary_dim == 4
    bad = json.loads(json.dumps(src))
    bad["model_type"] = "llama"
    with pytest.raises(ValueError):
        Config.from_json(bad)
    bad = json.loads(json.dumps(src))
    bad["text_config"]["rope_parameters"]["rope_type"] = "yarn"
    with pytest.raises(ValueError):
        Config.from_json(bad)


def test_safetensors_bf16_decode(tmp_path, oracle):
    """BF16 tensors widen as bits << 16 (src/safetensors.jl:28-30), or stay
    their raw bits for a device-side widen."""
    import json
    import struct
    from qdc_b200.model import read_safetensors
    vals = np.array([1.0, -2.5, 3.1415927, 1e-3], np.float32)
    bits = oracle.bf16_encode(vals)
    header = json.dumps({"w": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}}).encode()
    path = tmp_path / "t.safetensors"
    path.write_bytes(struct.pack("<Q", len(header)) + header + bits.tobytes())
    got = read_safetensors(str(path))["w"]
    assert np.array_equal(got.reshape(-1), oracle.bf16_decode(bits))
    raw = read_safetensors(str(path), raw_bf16=True)["w"]
    assert raw.dtype == np.uint16 and raw.shape == (2, 2)
    assert np.array_equal(raw.reshape(-1), bits)


@pytest.mark.parametrize("trim", [None, False, True, "env"])
def test_batch_backbone_hidden_left_padded_rows(cpu_backbone, monkeypatch, trim):
    """The batched hook (src/backbone.jl:66-70): each row's last-position
    state, rows left-padded by different amounts and by a common prefix,
    against the untrimmed single-sequence oracle forward of each row.  The
    common prefix is kept by default, as the reference's CUDA extension
    does (ext/QwenDecisionCoreCUDAExt.jl:12-20), and trimmed
    (src/backbone.jl:44-51) with trim_padding=True or
    QDC_B200_TRIM_PADDING=1."""
    import qdc_b200
    from oracle import forward as F
    from qdc_b200 import backbone as BB
    from qdc_b200.model import load_weights
    monkeypatch.setenv("QDC_B200_GRAPH", "0")
    monkeypatch.delenv("QDC_B200_TRIM_PADDING", raising=False)
    if trim == "env":
        monkeypatch.setenv("QDC_B200_TRIM_PADDING", "1")
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    seen = []
    real = BB.QwenBackbone.host_hidden
    monkeypatch.setattr(BB.QwenBackbone, "host_hidden",
                        lambda self, ids, mask=None, last_only=False:
                        seen.append(np.asarray(ids).shape) or real(self, ids, mask, last_only))
    S = 40
    ids = np.array([(np.arange(S) * (5 + r)) % 64 for r in range(3)])
    mask = np.ones((3, S), np.int64)
    for r, pad in enumerate((4, 9, 6)):
        mask[r, :pad] = 0
    mask[2, 20] = 0  # a hole inside a row as well
    kw = {} if trim in (None, "env") else {"trim_padding": trim}
    out = qdc_b200.batch_backbone_hidden(model, ids, mask, **kw)
    assert out.shape == (3, cfg.hidden)
    trimmed = trim in (True, "env")
    assert seen == [(3, S - 4 if trimmed else S)]
    om = F.load_model(GOLDEN)
    for r in range(3):
        expected = F.backbone_hidden(om, ids[r], mask[r])[-1]
        assert np.all(np.abs(out[r] - expected) <= 2e-5 + 2e-5 * np.abs(expected))
    assert qdc_b200.backbone.sequence_start(mask[0]) == 4
    assert qdc_b200.backbone.sequence_start(np.zeros(5)) == 4
    with pytest.raises(qdc_b200.ArgumentError):
        qdc_b200.batch_backbone_hidden(model, ids, mask[:, :-1])


def test_graph_cache_is_bounded(cpu_backbone, monkeypatch):
    """At most MAX_GRAPHS captured last-token forwards per model, least
    recently used evicted first (the capture itself is replaced by a stub
    here: capturing needs a GPU)."""
    from qdc_b200 import backbone as BB
    from qdc_b200.model import load_weights
    made = []

    class Stub:
        def __init__(self, model, B, S, full):
            self.graph, self.key = object(), (B, S, full)
            self.generation = model.ws.generation
            made.append(self.key)

        def __call__(self, ids, mask):
            return np.zeros((ids.shape[0], 8), np.float32)

    monkeypatch.setattr(BB, "_GraphedLastHidden", Stub)
    monkeypatch.setattr(BB, "MAX_GRAPHS", 3)
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    model._graphs = BB.collections.OrderedDict()
    for n in (5, 6, 7, 5, 8):
        model.last_hidden_graphed(np.ones((1, n), np.int64), np.ones((1, n), np.int64))
    assert list(model._graphs) == [(1, 7, True), (1, 5, True), (1, 8, True)]
    assert made == [(1, 5, True), (1, 6, True), (1, 7, True), (1, 8, True)]


def test_workspace_slots_repeat_by_call_order(cpu_backbone):
    """Every intermediate of the forward is a workspace slot: layers of one
    kind carve the same slots (each layer releases its slots when it ends),
    a second forward of the same shape carves exactly the slots of the
    first, and the forward never goes past the bytes forward_bytes planned
    (the workspace double asserts that on every take)."""
    from qdc_b200.model import Config, random_weights
    cfg = Config(hidden=64, head_dim=32, heads=4, kv_heads=2, key_heads=2, value_heads=4, key_dim=16,
                 value_dim=16, eps=1e-6, rope_theta=1e7, rotary_dim=8, vocab=128, intermediate=96,
                 layer_types=["linear_attention"] * 3 + ["full_attention"] * 2)
    model = cpu_backbone(cfg, {k: v.numpy() for k, v in random_weights(cfg, 1).items()})
    ids = np.arange(2 * 70).reshape(2, 70) % 128
    mask = np.ones((2, 70), np.int64)
    mask[1, :5] = 0
    model.batch_hidden(ids, mask)
    first = list(model.ws.takes)
    model.batch_hidden(ids[:, ::-1].copy(), mask)
    assert model.ws.takes == first
    assert model.ws.high <= model.ws.planned
    # root slots, then per layer: the three DeltaNet layers carve alike, as
    # do the two attention layers
    spans = {}
    for start, shape, dtype in first:
        spans.setdefault((shape, dtype), []).append(start)
    proj_delta = (2 * 70, cfg.qkv_width + cfg.value_width + 2 * cfg.value_heads)
    assert len(set(spans[(proj_delta, torch.float32)])) == 1 and len(spans[(proj_delta, torch.float32)]) == 3
    proj_full = (2 * 70, cfg.heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim)
    assert len(set(spans[(proj_full, torch.float32)])) == 1 and len(spans[(proj_full, torch.float32)]) == 2


def test_constant_caches_stay_bounded(cpu_backbone):
    """A model that sees many sequence lengths keeps at most MAX_CONSTS
    causal masks (each S x S on the device), least recently used evicted,
    and results do not depend on what was evicted."""
    import qdc_b200
    from qdc_b200 import backbone as BB
    from qdc_b200.model import load_weights
    cfg, w = load_weights(GOLDEN)
    model = cpu_backbone(cfg, w)
    first = qdc_b200.backbone_hidden(model, np.arange(5) % 64, np.ones(5, np.int64))
    for n in range(6, 6 + 2 * BB.MAX_CONSTS):
        qdc_b200.backbone_hidden(model, np.arange(n) % 64, np.ones(n, np.int64))
        assert len(model._const) <= BB.MAX_CONSTS
    assert ("upper", 5) not in model._const
    again = qdc_b200.backbone_hidden(model, np.arange(5) % 64, np.ones(5, np.int64))
    assert np.array_equal(again, first)
