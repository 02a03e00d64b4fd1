"""GPU: GatedDeltaNet2.forward_train_autograd (burn_gdn2.training on the
B200 kernels: chunked forward, gdn2_recurrent_bwd backward) against

  * the fused inference forward_train (same weights, same input): f32
    elementwise 1e-3 |ref| + 1e-3 RMS(ref);
  * float64 torch autograd of the same graph on the CPU with a plain-torch
    token-loop core (pinned to the oracle layer by test_training_cpu.py): the
    gradient of every weight and of the input.  f32 layers: elementwise
    1e-3 |ref| + 1e-3 RMS(ref) per tensor (gradient entries are sums over
    tokens and heads: entries near zero are cancellations at the RMS scale);
    bf16 layers: normwise 3e-2 per tensor (bf16 GEMMs and bf16 core inputs).
"""
import numpy as np
import pytest
import torch

from helpers import assert_close, assert_close_normwise
from training_ref import torch_loop_core

pytestmark = pytest.mark.gpu

CFGS = [
    (dict(hidden_size=256, num_heads=2, head_dim=128), 100),   # tensor-core chunk forward (K = 128)
    (dict(hidden_size=256, num_heads=2, head_dim=64), 100),    # CUDA-core chunk forward (K = 64)
    (dict(hidden_size=128, num_heads=1, head_dim=64, num_v_heads=2, allow_neg_eigval=True, min_decay=0.9), 70),
    (dict(hidden_size=256, num_heads=2, head_dim=64), 40),     # T <= 64: recurrent forward
]


def _f32_check(got, want, what):
    rms = float(np.sqrt(np.mean(want * want)))
    assert_close(got, want, rtol=1e-3, atol=1e-3 * rms, what=what)


def _layer(cfgd, dtype, gva="reference"):
    import burn_gdn2 as bg

    cfg = bg.Gdn2Config(mode=bg.Gdn2Mode.Chunk, chunk_size=64, **cfgd)
    return cfg, bg.GatedDeltaNet2.new(cfg, device="cuda", dtype=dtype, seed=41, gva_mode=gva)


@pytest.mark.parametrize("cfgd,T", CFGS)
def test_autograd_forward_matches_fused_forward(cfgd, T):
    cfg, m = _layer(cfgd, torch.float32)
    x = torch.randn(2, T, cfg.hidden_size, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():
        y = m.forward_train_autograd(x)
    ref = m.forward_train(x)
    _f32_check(y.cpu().numpy(), ref.cpu().numpy(), "autograd forward")


@pytest.mark.parametrize("cfgd,T", CFGS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_autograd_gradients_match_float64(cfgd, T, dtype):
    from burn_gdn2 import training

    cfg, m = _layer(cfgd, dtype)
    m.requires_grad_(True)
    gen = torch.Generator("cuda").manual_seed(4)
    x = torch.randn(2, T, cfg.hidden_size, device="cuda", generator=gen).to(dtype).requires_grad_(True)
    r = torch.randn(2, T, cfg.hidden_size, device="cuda", generator=gen)
    y = m.forward_train_autograd(x)
    (y.float() * r).sum().backward()
    P = m.parameters()

    P64 = {n: t.detach().double().cpu().requires_grad_(True) for n, t in P.items()}
    x64 = x.detach().double().cpu().requires_grad_(True)
    y64 = training.layer_forward(P64, cfg, x64, "reference", core=torch_loop_core)
    (y64 * r.double().cpu()).sum().backward()

    for n in P:
        got, want = P[n].grad.float().cpu().numpy(), P64[n].grad.numpy()
        if dtype == torch.float32:
            _f32_check(got, want, f"d{n}")
        else:
            assert_close_normwise(got, want, 3e-2, what=f"d{n}")
    gx, wx = x.grad.float().cpu().numpy(), x64.grad.numpy()
    if dtype == torch.float32:
        _f32_check(gx, wx, "dx")
    else:
        assert_close_normwise(gx, wx, 3e-2, what="dx")
