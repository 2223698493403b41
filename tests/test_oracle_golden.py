"""Pin the CPU oracle against the reference's own golden logits.

The reference checks its whole forward against PyTorch-computed logits of a
tiny Qwen3.5 checkpoint (test/backbone.jl:1-34, atol = rtol = 2e-5, probe
head test/runtests.jl:18-31).  oracle/forward.py runs that forward with every
norm / RoPE / gate / SwiGLU site going through the C oracle, so matching the
logits pins the oracle's per-layer ops.  The planted-mistake tests check the
pin is sensitive: each plants one plausible error in the oracle (on the CPU)
and the logits must then miss.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

TOL = 2e-5  # test/backbone.jl:10,24


def test_fixtures_match_manifest():
    """The committed fixtures are byte-for-byte the reference's
    (test/fixtures/native, SHA-256 recorded by tests/golden/make_golden.py)."""
    import hashlib
    with open(os.path.join(GOLDEN, "MANIFEST.json")) as f:
        manifest = json.load(f)
    files = [k for k in manifest if not k.startswith("_")]
    assert set(files) == {"config.json", "model.safetensors", "readout.safetensors", "reference.json",
                          "cuda_reference.json"}
    for name in files:
        with open(os.path.join(GOLDEN, name), "rb") as f:
            assert hashlib.sha256(f.read()).hexdigest() == manifest[name], name


@pytest.fixture(scope="module")
def model(oracle):
    from oracle import forward as F
    return F.load_model(GOLDEN)


@pytest.fixture(scope="module")
def readout():
    from oracle import forward as F
    return F.read_safetensors(os.path.join(GOLDEN, "readout.safetensors"))["weight"]


def _samples(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def _max_violation(model, readout, samples):
    from oracle import forward as F
    worst = 0.0
    for s in samples:
        expected = np.array(s["logits"], np.float64)
        actual = F.probe_logits(model, readout, s["inputs"]["input_ids"], s["inputs"]["attention_mask"])
        worst = max(worst, float((np.abs(actual - expected) / (TOL + TOL * np.abs(expected))).max()))
    return worst


def test_fixture_config(model):
    cfg = model.config
    # test/fixtures/native/config.json: rotary = head_dim * rope_parameters.partial_rotary_factor
    assert (cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.rotary_dim) == (8, 4, 2, 1, 4)
    assert cfg.layer_types == ["linear_attention", "full_attention"]


def test_reference_json_logits(model, readout):
    """All 5 samples (lengths 1/3/63/64/65, masks with holes) within 2e-5."""
    assert _max_violation(model, readout, _samples("reference.json")) <= 1.0


def test_cuda_reference_json_logits(model, readout):
    """The 21 x 3 rows beside it (lengths 1..256; prefix / holes / last-only
    masks).  No reference test loads this file, so it is an extra check."""
    assert _max_violation(model, readout, _samples("cuda_reference.json")) <= 1.0


def test_backbone_hidden_validation(model):
    from oracle import forward as F
    with pytest.raises(ValueError):
        F.backbone_hidden(model, [1, 2], [1])
    with pytest.raises(ValueError):
        F.backbone_hidden(model, [], [])
    with pytest.raises(ValueError):
        F.backbone_hidden(model, [64], [1])
    with pytest.raises(ValueError):
        F.backbone_hidden(model, [1, 2], [1, 2])


MUTATIONS = {
    # name -> (oracle function replaced, factory(original, oracle) -> replacement)
    "gated norm centered": (
        "gated_rms", lambda f, O: lambda o, z, w, eps: f(o, z, 1.0 + w, eps)),
    "gated norm without silu(z)": (
        "gated_rms", lambda f, O: lambda o, z, w, eps: (
            O.rms(o.reshape(-1, o.shape[-1]), w, eps, centered=False).reshape(o.shape[0], -1)
            * z.reshape(o.shape[0], -1))),
    "RoPE dropped": (
        "qk_norm_rope", lambda f, O: lambda x, w, eps, r, c, s, **k: f(x, w, eps, 0, c[:, :0], s[:, :0], **k)),
    "RoPE sign flipped": (
        "qk_norm_rope", lambda f, O: lambda x, w, eps, r, c, s, **k: f(x, w, eps, r, c, -s, **k)),
    "post norm uncentered": (
        "residual_rms", lambda f, O: lambda x, m, w, eps, **k: f(x, m, w, eps, centered=False)),
    "SwiGLU operands swapped": ("swiglu", lambda f, O: lambda g, u, **k: f(u, g, **k)),
    "RMS eps x1e6": ("rms", lambda f, O: lambda x, w, eps, **k: f(x, w, eps * 1e6, **k)),
}


@pytest.mark.parametrize("name", sorted(MUTATIONS))
def test_planted_mistake_is_caught(name, model, readout, oracle, monkeypatch):
    from oracle import forward as F
    attr, factory = MUTATIONS[name]
    monkeypatch.setattr(F.O, attr, factory(getattr(oracle, attr), oracle))
    assert _max_violation(model, readout, _samples("reference.json")) > 1.0
