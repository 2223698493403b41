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


@pytest.fixture
def cpu_backbone(monkeypatch, oracle):
    from qdc_b200 import backbone as BB
    from qdc_b200 import ops
    from qdc_b200.model import pack_layers

    n = lambda t: t.detach().cpu().numpy()
    c = lambda a: np.ascontiguousarray(a)
    T = lambda a: torch.from_numpy(c(a))

    def gather_rms(emb, ids, w, eps, ctx=None, **k):
        r, y = oracle.gather_rms(n(emb), np.asarray(ids, np.int32), None, n(w), eps)
        return T(r), T(y)

    def residual_rms(x, m, w, eps, ctx=None, **k):
        r, y = oracle.residual_rms(n(x), n(m), n(w), eps)
        return T(r), T(y)

    def residual_add_rms(r, m, w, eps, ctx=None, **k):
        rr, y = oracle.residual_rms(n(r), n(m), n(w), eps)
        r.copy_(T(rr))
        return r, T(y)

    def qk(x, w, eps, rot, cos, sin, pos_offset=0, seq_len=None, ctx=None, **k):
        return T(oracle.qk_norm_rope(c(n(x)), n(w), eps, rot, n(cos), n(sin), pos_offset=pos_offset,
                                     seq_len=seq_len))

    def q_k(qi, ki, wq, wk, eps, rot, cos, sin, seq_len=None, ctx=None, **k):
        return (T(oracle.qk_norm_rope(c(n(qi)), n(wq), eps, rot, n(cos), n(sin), seq_len=seq_len)),
                T(oracle.qk_norm_rope(c(n(ki)), n(wk), eps, rot, n(cos), n(sin), seq_len=seq_len)))

    def gated(o, z, w, eps, ctx=None, **k):
        # the kernel's layout contract: heads contiguous within a token
        assert o.stride(1) == o.shape[2] and z.stride(1) == z.shape[2]
        return T(oracle.gated_rms(c(n(o)), c(n(z)), n(w), eps))

    def swiglu(g, u, ctx=None, **k):
        return T(oracle.swiglu(c(n(g)), c(n(u)))[0]), None

    def conv_norm(proj, w, kh, kd, vh, vd, seq_len=None, ctx=None, **k):
        C = 2 * kh * kd + vh * vd
        q, kk, v = oracle.delta_conv_norm(c(n(proj))[:, :C], n(w).reshape(C, 4), kh, kd, vh, vd,
                                          seq_len=seq_len)
        return T(q), T(kk), T(v)

    def delta_gates(proj, start, heads, a_decay, dt_bias, ctx=None, **k):
        beta, decay = oracle.delta_gates(c(n(proj)), start, heads, n(a_decay), n(dt_bias))
        return T(beta), T(decay)

    def attn_gate(values, gate, ctx=None, **k):
        return T(oracle.attn_gate(c(n(values)), c(n(gate))))

    def rope_table(theta, r, rows, device=None):
        cs, sn = oracle.rope_table(theta, r, rows)
        return T(cs), T(sn)

    for name, fn in (("native_gather_rms", gather_rms), ("native_residual_rms", residual_rms),
                     ("native_residual_add_rms", residual_add_rms), ("native_q_k_norm_rope", q_k),
                     ("native_qk_norm_rope", qk),
                     ("native_gated_rms", gated), ("native_mlp_gate", swiglu),
                     ("native_delta_conv_norm", conv_norm), ("native_delta_gates", delta_gates),
                     ("native_attn_gate", attn_gate),
                     ("rope_table", rope_table)):
        monkeypatch.setattr(ops, name, fn)

    def make(config, weights):
        b = BB.QwenBackbone.__new__(BB.QwenBackbone)
        b.config, b.device, b.ctx = config, torch.device("cpu"), _Ctx()
        b.embedding = BB._device_f32(weights["embed_tokens.weight"], "cpu")
        b.final_norm = BB._device_f32(weights["norm.weight"], "cpu")
        b.layers, b._rope, b.trace = pack_layers(config, weights, "cpu"), {}, None
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


@pytest.mark.parametrize("scan", [True, False])
def test_chunked_delta_matches_token_recurrence(scan):
    """The chunked rule (zero-padded tail chunk), with the hand-off as a
    linear scan and per chunk, equals the token recurrence of
    src/backbone_cpu.jl:681-705 on odd lengths."""
    from qdc_b200.backbone import chunked_delta
    g = torch.Generator().manual_seed(0)
    for S in (1, 63, 64, 65, 130):
        B, Hk, Dk, Hv, Dv = 2, 2, 8, 4, 6
        q = torch.nn.functional.normalize(torch.randn(B, S, Hk, Dk, generator=g), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(B, S, Hk, Dk, generator=g), dim=-1)
        v = torch.randn(B, S, Hv, Dv, generator=g)
        beta = torch.rand(B, S, Hv, generator=g)
        decay = -torch.rand(B, S, Hv, generator=g)
        out = chunked_delta(q, k, v, beta, decay, Hv // Hk, scan=scan).double()
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
    real = BB.QwenBackbone.batch_hidden
    monkeypatch.setattr(BB.QwenBackbone, "batch_hidden",
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
