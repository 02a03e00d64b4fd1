"""GPU parity of the core backward (gdn2_recurrent_bwd) against the oracle's
adjoint (gdn2_oracle.fused_recurrent_backward, float64, itself pinned to
torch autograd and finite differences on the CPU), through the C ABI.

Tolerances.  f32 inputs: elementwise |d| <= 1e-3 |ref| + 1e-3 RMS(ref) per
gradient tensor.  Every gradient entry is a sum over the value columns and
the later tokens (dq, dk, db, dg) or over the key rows (dv, dw), so entries
near zero are cancellations whose f32 summation-order error sits at the
RMS scale, not at their own.  bf16 inputs (the oracle gets the same rounded
inputs and output gradient): the north-star bf16 criterion of
helpers.assert_close_bf16 (rel 2e-2 elementwise, floor 1e-2 RMS, normwise
1e-2 per head).
"""
import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import assert_close, assert_close_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"
NAMES = ("dq", "dk", "dv", "dg", "db", "dw", "dh0")


def _check(got, want, dtype, what):
    if dtype == torch.float32:
        rms = float(np.sqrt(np.mean(want * want)))
        assert_close(got, want, rtol=1e-3, atol=1e-3 * rms, what=what)
    else:
        assert_close_bf16(got, want, what=what)


def _case(B, Hq, HV, T, K, V, dtype, seed, with_state=True, with_dstate=True):
    a = O.make_core_inputs(B, HV, T, K, V, seed=seed, dtype=np.float32)
    rng = np.random.default_rng(seed + 1)
    keys = {n: a[n][:, :Hq] for n in "qkgb"}  # Hq key heads; value head hv reads key head hv // (HV // Hq)
    dev = {n: torch.tensor(x, dtype=torch.float32 if n == "g" else dtype, device=DEV) for n, x in keys.items()}
    for n in "vw":
        dev[n] = torch.tensor(a[n], dtype=dtype, device=DEV)
    dout = torch.tensor(rng.standard_normal((B, HV, T, V)).astype(np.float32), dtype=dtype, device=DEV)
    h0 = torch.tensor(0.3 * rng.standard_normal((B, HV, K, V)).astype(np.float32), device=DEV) if with_state else None
    dst = torch.tensor(0.5 * rng.standard_normal((B, HV, K, V)).astype(np.float32), device=DEV) if with_dstate else None
    return dev, dout, h0, dst


def _oracle(dev, dout, h0, dst, scale, HV):
    f = lambda t: t.detach().float().cpu().numpy().astype(np.float64)
    Hq = dev["q"].shape[1]
    rep = HV // Hq
    x = {n: np.repeat(f(dev[n]), rep, axis=1) for n in "qkgb"}
    B, _, T, K = x["q"].shape
    V = dev["v"].shape[3]
    s0 = f(h0) if h0 is not None else np.zeros((B, HV, K, V))
    ref = O.fused_recurrent_backward(x["q"], x["k"], f(dev["v"]), x["g"], x["b"], f(dev["w"]), s0, scale, f(dout),
                                     None if dst is None else f(dst))
    ref = list(ref)
    if rep > 1:  # key-side gradients of a shared key head sum over its group
        for i in (0, 1, 3, 4):
            ref[i] = ref[i].reshape(B, Hq, rep, T, K).sum(2)
    return ref


BWD_SHAPES = [
    # B, Hq, HV, T, K, V
    (1, 2, 2, 37, 128, 128),    # partial last sub-chunk; 8-CTA cluster per chain
    (2, 2, 2, 64, 64, 64),
    (1, 1, 1, 130, 32, 48),     # 3-CTA cluster, K = 32
    (1, 2, 2, 40, 128, 256),    # 512-thread CTAs
    (1, 1, 3, 24, 96, 16),      # GVA (key heads grouped), one CTA per chain, K = 96
    (2, 1, 1, 1, 128, 128),     # one token
]


@pytest.mark.parametrize("shape", BWD_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_recurrent_backward_matches_oracle(shape, dtype):
    import burn_gdn2 as bg

    B, Hq, HV, T, K, V = shape
    dev, dout, h0, dst = _case(B, Hq, HV, T, K, V, dtype, seed=21)
    scale = K ** -0.5
    got = bg.recurrent_backward(dev["q"], dev["k"], dev["v"], dev["g"], dev["b"], dev["w"], h0, scale, dout, dst)
    torch.cuda.synchronize()
    ref = _oracle(dev, dout, h0, dst, scale, HV)
    for name, x, r in zip(NAMES, got, ref):
        _check(x.cpu().numpy(), r, dtype, f"{name} {shape}")


def test_recurrent_backward_no_state_no_final_grad():
    import burn_gdn2 as bg

    dev, dout, _, _ = _case(1, 2, 2, 50, 128, 128, torch.float32, seed=5, with_state=False, with_dstate=False)
    got = bg.recurrent_backward(dev["q"], dev["k"], dev["v"], dev["g"], dev["b"], dev["w"], None, 0.1, dout, None)
    ref = _oracle(dev, dout, None, None, 0.1, 2)
    for name, x, r in zip(NAMES, got, ref):
        _check(x.cpu().numpy(), r, torch.float32, name)


def test_recurrent_backward_config2_head_length():
    """The config-2 head shape (K = V = 128) over T = 1024 tokens, one chain per value head."""
    import burn_gdn2 as bg

    dev, dout, h0, dst = _case(1, 2, 2, 1024, 128, 128, torch.float32, seed=8)
    got = bg.recurrent_backward(dev["q"], dev["k"], dev["v"], dev["g"], dev["b"], dev["w"], h0, 128 ** -0.5, dout,
                                dst)
    ref = _oracle(dev, dout, h0, dst, 128 ** -0.5, 2)
    for name, x, r in zip(NAMES, got, ref):
        _check(x.cpu().numpy(), r, torch.float32, name)


@pytest.mark.parametrize("T", [40, 200])
def test_gated_delta_core_autograd(T):
    """GatedDeltaCore: forward on the chunked (T > 64) or recurrent kernels,
    backward on gdn2_recurrent_bwd, driven by torch autograd; gradients of a
    loss on both outputs against the oracle's adjoint."""
    import burn_gdn2 as bg

    dev, dout, h0, dst = _case(1, 2, 2, T, 128, 128, torch.float32, seed=13)
    leaves = {n: t.clone().requires_grad_(True) for n, t in dev.items()}
    s0 = h0.clone().requires_grad_(True)
    out, st = bg.GatedDeltaCore.apply(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["b"], leaves["w"],
                                      s0, 128 ** -0.5, 64)
    ((out * dout).sum() + (st * dst).sum()).backward()
    ref = _oracle(dev, dout, h0, dst, 128 ** -0.5, 2)
    got = [leaves[n].grad for n in "qkvgbw"] + [s0.grad]
    order = ["dq", "dk", "dv", "dg", "db", "dw", "dh0"]
    for name, x, r in zip(order, got, ref):
        _check(x.cpu().numpy(), r, torch.float32, f"{name} T={T}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_recurrent_backward_unaligned_views(dtype):
    """Inputs that are column slices at an odd element offset (not on a 16-byte
    boundary): the kernel reads them synchronously instead of by cp.async."""
    import burn_gdn2 as bg

    B, HV, T, K, V = 1, 2, 45, 64, 32
    dev, dout, h0, dst = _case(B, HV, HV, T, K, V, dtype, seed=17)
    wide = {}
    for n, t in dev.items():
        w = torch.zeros(*t.shape[:3], t.shape[3] + 3, dtype=t.dtype, device=DEV)
        w[..., 1:1 + t.shape[3]] = t
        wide[n] = w[..., 1:1 + t.shape[3]]
    assert wide["q"].data_ptr() % 16 != 0
    got = bg.recurrent_backward(wide["q"], wide["k"], wide["v"], wide["g"], wide["b"], wide["w"], h0, 0.125, dout,
                                dst)
    ref = _oracle(dev, dout, h0, dst, 0.125, HV)
    for name, x, r in zip(NAMES, got, ref):
        _check(x.cpu().numpy(), r, dtype, f"{name} unaligned")


TRAJ_SHAPES = [
    # B, HV, T, K, V, chunk
    (1, 2, 200, 128, 128, 64),   # partial last chunk
    (2, 1, 37, 64, 48, 16),      # partial last sub-chunk, 3-CTA slices
    (1, 2, 5, 128, 256, 64),     # shorter than one sub-chunk
]


@pytest.mark.parametrize("shape", TRAJ_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_chunk_trajectory_matches_oracle(shape, dtype):
    """gdn2_chunk_trajectory: the state entering every chunk and v_new per token
    against the oracle's restatement of the crate's trajectory export."""
    import burn_gdn2 as bg

    B, HV, T, K, V, C = shape
    dev, _, h0, _ = _case(B, HV, HV, T, K, V, dtype, seed=9)
    states, vnew = bg.chunk_trajectory(dev["q"], dev["k"], dev["v"], dev["g"], dev["b"], dev["w"], h0, C)
    f = lambda t: t.detach().float().cpu().numpy().astype(np.float64)
    want_s, want_v = O.fused_recurrent_trajectory(*(f(dev[n]) for n in "qkvgbw"), f(h0), C)
    assert states.shape == want_s.shape
    _check(states.cpu().numpy(), want_s, dtype, f"states {shape}")
    _check(vnew.cpu().numpy(), want_v, dtype, f"v_new {shape}")
    s2, none = bg.chunk_trajectory(dev["q"], dev["k"], dev["v"], dev["g"], dev["b"], dev["w"], None, C,
                                   with_v_new=False)
    assert none is None and float(s2[:, :, 0].abs().max()) == 0.0  # zero initial state
