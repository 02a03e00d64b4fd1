"""GPU parity of gdn2_project_activations (the elementwise part of project,
src/module.rs:381-498) against the CPU oracle's own steps: short_conv_1d
(src/short_conv.rs:22-65), SiLU, l2_normalize_4d (src/l2norm.rs:13-16),
sigmoid gates and the softplus decay with the min_decay remap.

Raw inputs are column slices of one wider buffer, the way the module's
concatenated projection GEMM hands them over.  Tolerances: f32 rel 1e-3 /
abs 1e-4; bf16 by the bf16 criterion on bf16-rounded raw inputs.
"""
import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import F32_TOL, assert_close, assert_close_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"

CASES = [
    # B, T, H, K, HV, V, conv, cache, negeig, min_decay
    (2, 100, 2, 128, 2, 128, True, False, False, None),
    (1, 70, 4, 64, 4, 64, True, True, False, None),
    (2, 33, 2, 128, 4, 256, True, True, True, 0.9),
    (1, 65, 1, 256, 1, 128, True, False, False, None),
    (1, 40, 3, 32, 3, 48, False, False, True, None),
    (1, 2, 2, 128, 2, 128, True, True, False, None),
    # full 64-token blocks of 256-channel slices: the wide kernel (K = 32 .. 256),
    # with and without conv / cache; the T = 100 and 70 cases above split into a
    # wide block and a generic ragged tail
    (1, 128, 4, 64, 2, 128, True, True, True, 0.9),
    (2, 192, 2, 128, 2, 256, True, False, False, None),
    (1, 64, 2, 256, 2, 128, True, True, False, None),
    (1, 64, 8, 32, 4, 64, True, False, True, None),
    (1, 128, 2, 128, 2, 128, False, False, False, 0.5),
]


def _run(case, dtype, seed):
    import burn_gdn2 as bg

    B, T, H, K, HV, V, conv, cache, negeig, min_decay = case
    kd, vd = H * K, HV * V
    rng = np.random.default_rng(seed)
    widths = [kd, kd, vd, kd, vd, kd]
    ld = sum(widths) + 8  # wider than the slices: row stride != width
    buf = (rng.standard_normal((B * T, ld)) * 1.5).astype(np.float32)
    buf[:, sum(widths[:5]):sum(widths)] = rng.uniform(-9, 3, (B * T, kd))  # f raw: softplus both sides of 0
    dbuf = torch.tensor(buf, dtype=dtype, device=DEV)
    offs = np.cumsum([0] + widths)
    raws = [dbuf[:, offs[i]:offs[i] + widths[i]] for i in range(6)]
    conv_w = [rng.uniform(-0.5, 0.5, (n, 4)).astype(np.float32) for n in (kd, kd, vd)]
    conv_in = [rng.standard_normal((B, 3, n)).astype(np.float32) for n in (kd, kd, vd)] if cache else None
    a_log = rng.uniform(0.0, np.log(16.0), H).astype(np.float32)
    dt_bias = rng.uniform(-7, -2, kd).astype(np.float32)
    decay = rng.uniform(-1, 3, kd).astype(np.float32)
    t = lambda a: torch.tensor(a, device=DEV)
    (q, k, v, b, w, g), cout = bg.project_activations(
        *raws, batch=B, num_heads=H, head_k_dim=K, num_v_heads=HV, head_v_dim=V, a_log=t(a_log),
        dt_bias=t(dt_bias), conv_w=[t(x) for x in conv_w] if conv else None,
        conv_in=[t(x) for x in conv_in] if conv_in is not None else None, allow_neg_eigval=negeig,
        min_decay=min_decay, decay_factors=t(decay))
    torch.cuda.synchronize()
    # oracle on the same (dtype-rounded) raw values
    r64 = [x.float().cpu().numpy().astype(np.float64).reshape(B, T, -1) for x in raws]
    if conv:
        outs = [O.short_conv_1d(r64[i], conv_w[i].astype(np.float64),
                                None if conv_in is None else conv_in[i].astype(np.float64)) for i in range(3)]
        qa, ka, va = (o[0] for o in outs)
        caches = [o[1] for o in outs]
    else:
        qa, ka, va = (O.silu(r64[i]) for i in range(3))
        caches = None
    q4 = O.l2_normalize_4d(qa.reshape(B, T, H, K), 1e-6).reshape(B, T, kd)
    k4 = O.l2_normalize_4d(ka.reshape(B, T, H, K), 1e-6).reshape(B, T, kd)
    b_ref = O.sigmoid(r64[3]) * (2.0 if negeig else 1.0)
    w_ref = O.sigmoid(r64[4])
    g_ref = -np.repeat(np.exp(a_log.astype(np.float64)), K) * O.softplus(r64[5] + dt_bias)
    if min_decay is not None:
        fac = O.sigmoid(decay.astype(np.float64)) * (1.0 - min_decay)
        g_ref = np.log(fac * np.exp(g_ref) + min_decay)
    got = {n: x.float().cpu().numpy().reshape(B, T, -1) for n, x in zip("qkvbwg", (q, k, v, b, w, g))}
    want = dict(q=q4, k=k4, v=va, b=b_ref, w=w_ref, g=g_ref)
    for n in "qkvbwg":
        if dtype == torch.float32 or n == "g":
            assert_close(got[n], want[n], what=n, **F32_TOL)
        else:
            assert_close_bf16(got[n], want[n], what=n)
    if conv:
        for i, n in enumerate("qkv"):
            assert_close(cout[i].cpu().numpy(), caches[i], what=f"cache {n}", rtol=0, atol=0)
    else:
        assert cout is None


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_project_activations_matches_oracle(case, dtype):
    _run(case, dtype, seed=101 + CASES.index(case))


def test_decay_softplus_accuracy():
    """g = -exp(A_log) softplus(f + dt_bias) over f from -40 to 40 (both
    branches of the kernel's softplus, the series for e^x < 1/8 and the
    base-2 logarithm above, and the x > 20 cut) within 1e-5 relative of
    numpy's log(1 + e^x)."""
    import burn_gdn2 as bg

    H, K = 1, 128
    f = np.linspace(-40.0, 40.0, 64 * K).astype(np.float32).reshape(64, K)
    dev = lambda a: torch.tensor(a, device=DEV)
    raw = dev(np.zeros((64, K), np.float32))
    (_, _, _, _, _, g), _ = bg.project_activations(
        raw, raw, raw, raw, raw, dev(f), batch=1, num_heads=H, head_k_dim=K, num_v_heads=H, head_v_dim=K,
        a_log=dev(np.zeros(H, np.float32)), dt_bias=dev(np.zeros(K, np.float32)))
    want = -np.logaddexp(0.0, f.astype(np.float64))
    assert_close(g.cpu().numpy(), want, rtol=1e-5, atol=1e-30, what="softplus")
