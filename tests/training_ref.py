"""Test-side reference core for the differentiable layer: the token recurrence
(src/kernel/fused_recurrent.rs:11-56) as plain torch ops, so torch autograd
differentiates it exactly (float64 on the CPU).  Checker only."""
import torch


def torch_loop_core(q, k, v, g, b, w, scale, chunk):
    B, HV, T, K = q.shape
    S = torch.zeros(B, HV, K, v.shape[3], dtype=q.dtype)
    outs = []
    for t in range(T):
        S = S * torch.exp(g[:, :, t])[..., None]
        e = (S * (b[:, :, t] * k[:, :, t])[..., None]).sum(2)
        u = w[:, :, t] * v[:, :, t] - e
        S = S + k[:, :, t, :, None] * u[:, :, None, :]
        outs.append(scale * (S * q[:, :, t, :, None]).sum(2))
    return torch.stack(outs, 2), S
