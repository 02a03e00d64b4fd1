"""CPU: the oracle's adjoint of the token recurrence
(gdn2_oracle.fused_recurrent_backward) pinned two ways, since the reference
has no wired backward to take vectors from (the crate trains through burn
autodiff of src/forward.rs:44-278):

  * against torch autograd (float64) of the same recurrence written in torch
    (src/kernel/fused_recurrent.rs:11-56), every input gradient, with an
    initial state and a final-state gradient, to 1e-10;
  * against central finite differences of the oracle's own forward on a few
    coordinates of every input, to 1e-6.
"""
import numpy as np
import pytest
import torch

import gdn2_oracle as O


def _inputs(seed, B=2, H=2, T=13, K=8, V=6):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, T, K))
    kr = rng.standard_normal((B, H, T, K))
    k = kr / np.sqrt((kr * kr).sum(-1, keepdims=True))
    v = rng.standard_normal((B, H, T, V))
    g = rng.uniform(-0.4, -0.01, (B, H, T, K))
    b = rng.uniform(0.0, 2.0, (B, H, T, K))
    w = rng.uniform(0.2, 1.0, (B, H, T, V))
    h0 = 0.3 * rng.standard_normal((B, H, K, V))
    dout = rng.standard_normal((B, H, T, V))
    dst = 0.5 * rng.standard_normal((B, H, K, V))
    return q, k, v, g, b, w, h0, dout, dst


def _torch_forward(q, k, v, g, b, w, h0, scale):
    S = h0
    outs = []
    for t in range(q.shape[2]):
        S = S * torch.exp(g[:, :, t])[..., None]
        e = (S * (b[:, :, t] * k[:, :, t])[..., None]).sum(2)
        u = w[:, :, t] * v[:, :, t] - e
        S = S + k[:, :, t, :, None] * u[:, :, None, :]
        outs.append(scale * (S * q[:, :, t, :, None]).sum(2))
    return torch.stack(outs, 2), S


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_backward_matches_torch_autograd(seed):
    q, k, v, g, b, w, h0, dout, dst = _inputs(seed)
    scale = 0.35
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v, g, b, w, h0)]
    o, S = _torch_forward(*ts, scale)
    (o * torch.tensor(dout)).sum().add_((S * torch.tensor(dst)).sum()).backward()
    ref = [t.grad.numpy() for t in ts]
    got = O.fused_recurrent_backward(q, k, v, g, b, w, h0, scale, dout, dst)
    for name, r, x in zip(("dq", "dk", "dv", "dg", "db", "dw", "dh0"), ref, got):
        assert np.abs(r - x).max() <= 1e-10 * max(1.0, np.abs(r).max()), name


def test_oracle_backward_matches_finite_differences():
    q, k, v, g, b, w, h0, dout, dst = _inputs(3, B=1, H=1, T=7, K=4, V=3)
    scale = 0.5
    args = [q, k, v, g, b, w, h0]

    def loss(a):
        o, S = O.fused_recurrent_forward(a[0], a[1], a[2], a[3], a[4], a[5], a[6], scale)
        return float((o * dout).sum() + (S * dst).sum())

    grads = O.fused_recurrent_backward(q, k, v, g, b, w, h0, scale, dout, dst)
    rng = np.random.default_rng(4)
    eps = 1e-6
    for i, x in enumerate(args):
        for _ in range(4):
            idx = tuple(int(rng.integers(0, n)) for n in x.shape)
            plus = [a.copy() for a in args]
            minus = [a.copy() for a in args]
            plus[i][idx] += eps
            minus[i][idx] -= eps
            fd = (loss(plus) - loss(minus)) / (2 * eps)
            assert abs(fd - grads[i][idx]) <= 1e-6 * max(1.0, abs(fd)), (i, idx, fd, grads[i][idx])


def test_oracle_trajectory_matches_forward_prefixes():
    """The exported chunk-start states are the forward's final states of the
    prefixes, and v_new reproduces the output: o_t = scale q_t^T S_t with
    S_t = e^{g_t} S_{t-1} + k_t v_new_t^T."""
    q, k, v, g, b, w, h0, _, _ = _inputs(7, T=21)
    C = 8
    states, vnew = O.fused_recurrent_trajectory(q, k, v, g, b, w, h0, C)
    assert states.shape[2] == 3
    assert np.abs(states[:, :, 0] - h0).max() == 0.0
    for i in range(1, 3):
        _, S = O.fused_recurrent_forward(q[:, :, :i * C], k[:, :, :i * C], v[:, :, :i * C], g[:, :, :i * C],
                                         b[:, :, :i * C], w[:, :, :i * C], h0, 1.0)
        assert np.abs(states[:, :, i] - S).max() <= 1e-12
    o, _ = O.fused_recurrent_forward(q, k, v, g, b, w, h0, 0.5)
    S = h0.copy()
    for t in range(q.shape[2]):
        S = S * np.exp(g[:, :, t])[..., None] + k[:, :, t, :, None] * vnew[:, :, t, None, :]
        assert np.abs(0.5 * (S * q[:, :, t, :, None]).sum(2) - o[:, :, t]).max() <= 1e-12
