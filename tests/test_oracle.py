"""CPU: the oracle against the reference's golden vectors and the
reference's own algebraic tests (re-expressed on the numpy restatement).

Pins (tolerances are the reference's):
  * tests/gen_reference.py layer outputs, the stream tests/bit_exact.rs
    checks at 5e-4 (fixtures in tests/golden/, made by gen_golden.py);
  * tests/stable_chunk.rs:11-72  chunk (16, 64) == per-token, 1e-3;
  * tests/test_chunk.rs:200-256  T=130 partial chunk, real decay, 1e-4;
  * tests/autodiff.rs:31-149     decode == full forward (1e-6),
    prefill -> decode handoff (1e-6), chunk == fused (1e-4).
"""
import numpy as np
import pytest

import gdn2_oracle as O
from helpers import load_golden

GOLDEN_SETS = ["ref_d64.npz", "ref_d64_negeig.npz", "ref_d256_k64.npz"]


@pytest.mark.parametrize("name", GOLDEN_SETS)
@pytest.mark.parametrize("mode", ["fused_recurrent", "chunk"])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_oracle_matches_reference_golden(name, mode, dtype):
    cfgd, weights, cases = load_golden(name)
    cfg = O.Gdn2Config(mode=mode, **cfgd)
    layer = O.Gdn2Layer(cfg, weights, dtype)
    worst = 0.0
    for x, y in cases:
        out, _ = layer.forward(x.astype(dtype), None, True)
        worst = max(worst, float(np.abs(out - y).max()))
    assert worst < 5e-4, worst  # tests/bit_exact.rs:11


def _stable_inputs(rng, decay, B=2, H=3, T=96, K=8, V=8):
    q = rng.standard_normal((B, H, T, K))
    kr = rng.standard_normal((B, H, T, K))
    k = kr / np.sqrt((kr * kr).sum(-1, keepdims=True))
    v = rng.standard_normal((B, H, T, V))
    g = rng.uniform(decay[0], decay[1], (B, H, T, 1))
    b = rng.uniform(0.0, 1.0, (B, H, T, 1))
    w = rng.standard_normal((B, H, T, V))
    return q, k, v, g, b, w


@pytest.mark.parametrize("decay", [(-0.3, -0.02), (-5.0, -0.5)])
def test_stable_chunk(decay):
    """tests/stable_chunk.rs:11-72 (scalar-broadcast g, b; scale 1)."""
    rng = np.random.default_rng(1)
    q, k, v, g, b, w = (x.astype(np.float32) for x in _stable_inputs(rng, decay))
    s0 = np.zeros((2, 3, 8, 8), np.float32)
    o_ref, s_ref = O.fused_recurrent_forward(q, k, v, g, b, w, s0, 1.0)
    for c in (16, 64):
        o, s = O.chunk_wy_forward(q, k, v, g, b, w, s0, 1.0, c)
        assert np.abs(o - o_ref).max() < 1e-3
        assert np.abs(s - s_ref).max() < 1e-3


def test_chunk_matches_fused_with_real_decay():
    """tests/test_chunk.rs:200-256: per-channel decay, T=130, random S0."""
    rng = np.random.default_rng(2)
    B, H, T, K, V = 2, 3, 130, 16, 8
    g = rng.uniform(-0.15, -0.01, (B, H, T, K))
    q = rng.standard_normal((B, H, T, K))
    kr = rng.standard_normal((B, H, T, K))
    k = kr / np.sqrt((kr ** 2).sum(-1, keepdims=True))
    v = rng.standard_normal((B, H, T, V))
    e = rng.uniform(0.0, 1.0, (B, H, T, K))
    w = rng.standard_normal((B, H, T, V))
    s0 = rng.standard_normal((B, H, K, V))
    args = [x.astype(np.float32) for x in (q, k, v, g, e, w, s0)]
    oc, sc = O.chunk_wy_forward(*args, 0.125, 64)
    of, sf = O.fused_recurrent_forward(*args, 0.125)
    assert np.abs(oc - of).max() < 1e-4
    assert np.abs(sc - sf).max() < 1e-4


@pytest.mark.parametrize("use_sc", [True, False])
def test_decode_equals_full_forward(use_sc):
    """tests/autodiff.rs:31-66: token-by-token with state == one pass."""
    cfg = O.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16, use_short_conv=use_sc)
    layer = O.Gdn2Layer(cfg, O.init_weights(cfg, seed=3), np.float64)
    x = np.random.default_rng(4).standard_normal((2, 12, 32))
    full, _ = layer.forward(x, None, True)
    st = None
    outs = []
    for t in range(12):
        y, st = layer.forward(x[:, t:t + 1], st, True)
        outs.append(y)
    assert np.abs(np.concatenate(outs, 1) - full).max() < 1e-6


def test_prefill_then_decode():
    """tests/autodiff.rs:70-104."""
    cfg = O.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16)
    layer = O.Gdn2Layer(cfg, O.init_weights(cfg, seed=5), np.float64)
    x = np.random.default_rng(6).standard_normal((1, 9, 32))
    full, _ = layer.forward(x, None, True)
    _, st = layer.forward(x[:, :8], None, True)
    nxt, _ = layer.forward(x[:, 8:9], st, True)
    assert np.abs(nxt - full[:, 8:9]).max() < 1e-6


def test_chunk_and_fused_agree_projected():
    """tests/autodiff.rs:108-149: chunk (C=16) vs per-token on projected inputs."""
    cfg = O.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16, mode="chunk")
    layer = O.Gdn2Layer(cfg, O.init_weights(cfg, seed=7), np.float32)
    x = np.random.default_rng(8).standard_normal((1, 80, 32)).astype(np.float32)
    p, _ = layer.project(x)
    s0 = np.zeros((1, 2, 16, 16), np.float32)
    oc, _ = O.chunk_wy_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], s0, 16 ** -0.5, 16)
    of, _ = O.fused_recurrent_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], s0, 16 ** -0.5)
    assert np.abs(oc - of).max() < 1e-4


def test_gva_repeat_reference_layout():
    """src/module.rs:457-468: value head h*rep+j at time t reads key-side
    token (j*T + t) // rep (H=2, T=4, rep=2 -> [[0,0,1,1],[2,2,3,3],...])."""
    B, H, T, K, rep = 1, 2, 4, 1, 2
    x = np.arange(H * T, dtype=np.float64).reshape(B, H, T, K) % T
    r = O.gva_repeat_ref(x, rep)[0, :, :, 0]
    assert r.tolist() == [[0, 0, 1, 1], [2, 2, 3, 3], [0, 0, 1, 1], [2, 2, 3, 3]]


def test_config_validate_messages():
    """src/config.rs:71-111."""
    O.Gdn2Config().validate()
    for bad in (dict(hidden_size=0), dict(expand_v=1.3), dict(num_v_heads=8), dict(num_v_heads=24),
                dict(chunk_size=0), dict(norm_eps=0.0)):
        with pytest.raises(ValueError):
            O.Gdn2Config(**bad).validate()


def test_min_decay_bounds_decay():
    """src/module.rs:430-440: exp(g) >= min_decay after the remap."""
    cfg = O.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16, min_decay=0.9)
    layer = O.Gdn2Layer(cfg, O.init_weights(cfg, seed=9), np.float64)
    p, _ = layer.project(np.random.default_rng(10).standard_normal((1, 20, 32)) * 5)
    assert np.exp(p["g"]).min() >= 0.9 - 1e-12
