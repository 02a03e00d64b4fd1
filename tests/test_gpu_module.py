"""GPU parity of the whole layer (burn_gdn2.GatedDeltaNet2 over the C ABI)
against the reference's golden vectors and the CPU oracle.

  * gen_reference.py fixtures, 5e-4 (tests/bit_exact.rs:11) — fused
    recurrent path (T <= 64) and chunk path (T > 64, mode Chunk);
  * decode token by token == full forward; prefill -> decode handoff
    (tests/autodiff.rs:31-104), at the north-star f32 tolerance;
  * GVA (reference repeat layout and grouped mode), min_decay, neg-eig, bf16.
"""
import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import BF16_RTOL, F32_TOL, assert_close, assert_close_normwise, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _module(cfgd, weights, mode, dtype=torch.float32, gva_mode="reference", **extra):
    import burn_gdn2 as bg

    cfg = bg.Gdn2Config(mode=mode, **cfgd, **extra)
    return bg.GatedDeltaNet2(cfg, weights, device=DEV, dtype=dtype, gva_mode=gva_mode)


@pytest.mark.parametrize("name", ["ref_d64.npz", "ref_d64_negeig.npz", "ref_d256_k64.npz"])
@pytest.mark.parametrize("mode", ["FusedRecurrent", "Chunk"])
def test_layer_matches_reference_golden(name, mode):
    import burn_gdn2 as bg

    cfgd, weights, cases = load_golden(name)
    m = _module(cfgd, weights, getattr(bg.Gdn2Mode, mode))
    worst = 0.0
    for x, y in cases:
        out, _ = m.forward(torch.tensor(x, device=DEV), None, True)
        worst = max(worst, float(np.abs(out.cpu().numpy() - y).max()))
        out2 = m.forward_train(torch.tensor(x, device=DEV))
        worst = max(worst, float(np.abs(out2.cpu().numpy() - y).max()))
    assert worst < 5e-4, worst


@pytest.mark.parametrize("use_sc", [True, False])
def test_decode_equals_full_forward(use_sc):
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=32, num_heads=2, head_dim=16, use_short_conv=use_sc)
    ocfg = O.Gdn2Config(**cfgd)
    m = _module(cfgd, O.init_weights(ocfg, seed=3), bg.Gdn2Mode.FusedRecurrent)
    x = torch.tensor(np.random.default_rng(4).standard_normal((2, 12, 32)), dtype=torch.float32, device=DEV)
    full, _ = m.forward(x, None, True)
    st = None
    outs = []
    for t in range(12):
        y, st = m.forward(x[:, t:t + 1], st, True)
        outs.append(y)
    assert_close(torch.cat(outs, 1).cpu().numpy(), full.cpu().numpy(), what="decode", **F32_TOL)


def test_prefill_then_decode_chunk_prefill():
    """Prefill of 200 tokens (chunk path) then 3 decode steps == one pass."""
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=64, num_heads=2, head_dim=32)
    ocfg = O.Gdn2Config(**cfgd)
    W = O.init_weights(ocfg, seed=5)
    m = _module(cfgd, W, bg.Gdn2Mode.Chunk)
    x = np.random.default_rng(6).standard_normal((2, 203, 64)).astype(np.float32)
    layer = O.Gdn2Layer(O.Gdn2Config(mode="chunk", **cfgd), W, np.float64)
    full, _ = layer.forward(x.astype(np.float64), None, True)
    _, st = m.forward(torch.tensor(x[:, :200], device=DEV), None, True)
    for t in range(200, 203):
        y, st = m.forward(torch.tensor(x[:, t:t + 1], device=DEV), st, True)
        assert_close(y.cpu().numpy(), full[:, t:t + 1], what=f"decode {t}", **F32_TOL)


@pytest.mark.parametrize("T", [1, 20, 100])
@pytest.mark.parametrize("gva_mode", ["reference", "grouped"])
def test_gva_minDecay_negEig_vs_oracle(T, gva_mode):
    """BASELINE config-4 features (GVA H -> 2H, neg-eig, min_decay 0.9,
    expand_v 2) at small size, against the oracle in the same GVA mode."""
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=64, num_heads=2, head_dim=16, num_v_heads=4, expand_v=2.0, allow_neg_eigval=True,
                min_decay=0.9)
    ocfg = O.Gdn2Config(mode="chunk", **cfgd)
    W = O.init_weights(ocfg, seed=7)
    layer = O.Gdn2Layer(ocfg, W, np.float64, gva=gva_mode)
    x = np.random.default_rng(8).standard_normal((2, T, 64)).astype(np.float32)
    want, _ = layer.forward(x.astype(np.float64), None, True)
    m = _module(cfgd, W, bg.Gdn2Mode.Chunk, gva_mode=gva_mode)
    got, _ = m.forward(torch.tensor(x, device=DEV), None, True)
    assert_close(got.cpu().numpy(), want, what="forward", **F32_TOL)
    want_t = layer.forward_train(x.astype(np.float64))
    got_t = m.forward_train(torch.tensor(x, device=DEV))
    assert_close(got_t.cpu().numpy(), want_t, what="forward_train", **F32_TOL)


def test_gva_decode_inplace_cluster():
    """Decode with GVA: the conv caches of a key head are shared by its value
    heads and updated in place (cluster path); 6 steps == one pass."""
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=64, num_heads=2, head_dim=32, num_v_heads=8, expand_v=2.0)
    ocfg = O.Gdn2Config(**cfgd)
    W = O.init_weights(ocfg, seed=9)
    layer = O.Gdn2Layer(ocfg, W, np.float64)
    x = np.random.default_rng(10).standard_normal((3, 6, 64)).astype(np.float32)
    m = _module(cfgd, W, bg.Gdn2Mode.FusedRecurrent)
    st = None
    ost = None
    for t in range(6):
        y, st = m.forward(torch.tensor(x[:, t:t + 1], device=DEV), st, True)
        yo, ost = layer.forward(x[:, t:t + 1].astype(np.float64), ost, True)
        assert_close(y.cpu().numpy(), yo, what=f"step {t}", **F32_TOL)
    assert_close(st.recurrent.cpu().numpy(), ost.recurrent, what="state", **F32_TOL)
    assert_close(st.conv_q.cpu().numpy(), ost.conv_q, what="conv_q", **F32_TOL)


@pytest.mark.parametrize("mode", ["FusedRecurrent", "Chunk"])
def test_layer_bf16_vs_oracle(mode):
    """bf16 weights/activations with f32 accumulation vs the f64 oracle on
    the same bf16-rounded weights: rel 2e-2 normwise.  Every projection and
    activation of the layer is stored in bf16 (one rounding each), so an
    elementwise bound is only meaningful on the core kernels, which
    test_gpu_core checks elementwise."""
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=128, num_heads=2, head_dim=64)
    ocfg = O.Gdn2Config(mode="chunk" if mode == "Chunk" else "fused_recurrent", **cfgd)
    W = O.init_weights(ocfg, seed=11)
    Wb = {k: torch.tensor(v).to(torch.bfloat16).float().numpy() for k, v in W.items()}
    x = np.random.default_rng(12).standard_normal((2, 150, 128)).astype(np.float32)
    xb = torch.tensor(x).to(torch.bfloat16).float().numpy()
    want = O.Gdn2Layer(ocfg, Wb, np.float64).forward_train(xb.astype(np.float64))
    m = _module(cfgd, W, getattr(bg.Gdn2Mode, mode), dtype=torch.bfloat16)
    got = m.forward_train(torch.tensor(xb, device=DEV, dtype=torch.bfloat16))
    assert_close_normwise(got.float().cpu().numpy(), want, BF16_RTOL, what="bf16 layer")


@pytest.mark.parametrize("gva_mode", ["grouped", "reference"])
def test_multi_token_inplace_cluster_path(gva_mode):
    """T = 5 continuation with state (in-place conv caches shared by 2 value
    heads x 2 column slices: the cluster path of the multi-token kernel),
    K = 128, V = 256, after a 70-token chunked prefill; vs the oracle."""
    import burn_gdn2 as bg

    cfgd = dict(hidden_size=128, num_heads=2, head_dim=128, num_v_heads=4, expand_v=2.0)
    ocfg = O.Gdn2Config(mode="chunk", **cfgd)
    W = O.init_weights(ocfg, seed=13)
    layer = O.Gdn2Layer(ocfg, W, np.float64, gva=gva_mode)
    x = np.random.default_rng(14).standard_normal((2, 75, 128)).astype(np.float32)
    m = _module(cfgd, W, bg.Gdn2Mode.Chunk, gva_mode=gva_mode)
    _, st = m.forward(torch.tensor(x[:, :70], device=DEV), None, True)
    _, ost = layer.forward(x[:, :70].astype(np.float64), None, True)
    y, st = m.forward(torch.tensor(x[:, 70:], device=DEV), st, True)
    yo, ost = layer.forward(x[:, 70:].astype(np.float64), ost, True)
    assert_close(y.cpu().numpy(), yo, what="continuation", **F32_TOL)
    assert_close(st.recurrent.cpu().numpy(), ost.recurrent, what="state", **F32_TOL)
    for n in ("conv_q", "conv_k", "conv_v"):
        assert_close(getattr(st, n).cpu().numpy(), getattr(ost, n), what=n, **F32_TOL)


def test_graphed_calls_match_eager():
    """CUDA-graph replay (GraphedCall) of forward_train at BASELINE config 1
    (f32, K = 64: the CUDA-core chunk path) and of a decode step that
    updates Gdn2State in place: replays on new inputs copied into the static
    buffers give exactly the eager outputs and states."""
    import burn_gdn2 as bg

    cfg = bg.Gdn2Config(hidden_size=256, num_heads=4, head_dim=64, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    m = bg.GatedDeltaNet2.new(cfg, device=DEV, dtype=torch.float32, seed=0)
    g = torch.Generator(device=DEV).manual_seed(5)
    xs = [torch.randn(1, 1024, 256, generator=g, device=DEV) for _ in range(2)]
    xin = torch.empty_like(xs[0])
    gc = bg.GraphedCall(m.forward_train, xin)
    for x in xs:
        xin.copy_(x)
        y = gc.replay().clone()
        assert torch.equal(y, m.forward_train(x))
    # decode: the same prefill state in two copies, one advanced eagerly, one by graph replays
    _, st = m.forward(xs[0][:, :100], None, True)
    _, st2 = m.forward(xs[0][:, :100], None, True)
    tok = torch.empty(1, 1, 256, device=DEV)
    gd = bg.GraphedCall(lambda t: m.forward(t, st2, True)[0], tok, warmup=1)
    # the capture's warm-up advanced st2 by one step, the capture itself by none: replay from a fresh copy
    for name in ("recurrent", "conv_q", "conv_k", "conv_v"):
        getattr(st2, name).copy_(getattr(st, name))
    for i in range(3):
        t = xs[1][:, i:i + 1]
        tok.copy_(t)
        yg = gd.replay().clone()
        ye, st = m.forward(t, st, True)
        assert torch.equal(yg, ye)
        assert torch.equal(st2.recurrent, st.recurrent)
