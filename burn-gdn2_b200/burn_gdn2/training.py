"""Differentiable GatedDeltaNet2 forward for training.

The crate trains by burn autodiff of its tensor path: ``forward_train``
(src/module.rs:326-375) over ``project`` (src/module.rs:381-498), the chunked
core (src/forward.rs:44-278) and the gated RMS norm + o_proj
(src/module.rs:501-517).  ``layer_forward`` is the same graph for torch
autograd: the projections and every elementwise step are torch ops, the
recurrence is ``GatedDeltaCore`` (chunked tensor-core forward, exact-f32
backward kernel), so ``loss.backward()`` gives the gradient of every weight
and of the input.  The fused inference path (``GatedDeltaNet2.forward_train``)
stays the fast forward; this one keeps the intermediates autograd needs.

``layer_forward(params, cfg, x, gva_mode, core)`` works on any device and
dtype for its torch part; ``core`` computes (o [B,HV,T,V], final state) from
(q, k, v, g, b, w, scale, chunk) and is ``cuda_core`` for the product.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

import torch
import torch.nn.functional as F

from .config import Gdn2Config
from .ops import GatedDeltaCore

SHORT_CONV_KERNEL = 4  # src/short_conv.rs:5
SHORT_CONV_CACHE = 3  # src/short_conv.rs:7

# weights of one layer, the names of GatedDeltaNet2's constructor (projections stored [in, out])
PARAM_NAMES = ("q_proj", "k_proj", "v_proj", "f_proj_0", "f_proj_1", "b_proj", "w_proj", "g_proj_0", "g_proj_1_w",
               "g_proj_1_b", "A_log", "dt_bias", "o_norm_w", "o_proj", "q_conv_w", "k_conv_w", "v_conv_w")


def short_conv_silu(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Causal depthwise conv (kernel 4) + SiLU from a zero state: the sequence
    start padded by replicating token 0 three times (src/short_conv.rs:22-65).
    x [B,T,C]; weight [C,4].  One depthwise conv1d over the replicate-padded
    [B,C,T+3] sequence (cross-correlation: out[t] = sum_i w[c,i] x_pad[t+i])
    instead of four shifted products, so forward and backward are a few
    kernels, not a few dozen."""
    C = x.shape[2]
    xp = F.pad(x.transpose(1, 2), (SHORT_CONV_CACHE, 0), mode="replicate")
    out = F.conv1d(xp, weight.reshape(C, 1, SHORT_CONV_KERNEL), groups=C)
    return F.silu(out.transpose(1, 2).contiguous())


def l2_normalize(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(sum x^2 + eps) over the last dim (src/l2norm.rs:13-16)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gva_repeat(x: torch.Tensor, rep: int, gva_mode: str) -> torch.Tensor:
    """Key-side [B,H,T,K] -> [B,H*rep,T,K].  "reference": the crate's
    unsqueeze(3).repeat(..).reshape (src/module.rs:457-468), value head
    h*rep + j reads key token (j*T + t) // rep; "grouped": value head hv reads
    key head hv // rep at the same token."""
    B, H, T, K = x.shape
    if gva_mode == "reference":
        return x.unsqueeze(3).repeat(1, 1, 1, rep, 1).reshape(B, H * rep, T, K)
    return x.repeat_interleave(rep, dim=1)


def project(params: Dict[str, torch.Tensor], cfg: Gdn2Config, x: torch.Tensor, gva_mode: str, core_dtype):
    """src/module.rs:381-498 from a zero conv state.  Returns q, k, g, b
    [B,HV,T,K], v, w [B,HV,T,V] (q, k, v, b, w in core_dtype, g f32) and the
    gate [B,T,HV,V]; activations are computed in f32 or wider."""
    P = params
    h, hk, hv, vh = cfg.num_heads, cfg.head_dim, cfg.hv, cfg.v_head
    B, T, _ = x.shape
    kd = h * hk
    wide = torch.promote_types(P["A_log"].dtype, torch.float32)
    up = lambda t: t.to(wide)
    q_raw, k_raw, v_raw = up(x @ P["q_proj"]), up(x @ P["k_proj"]), up(x @ P["v_proj"])
    if cfg.use_short_conv:
        q_act = short_conv_silu(q_raw, P["q_conv_w"].to(wide))
        k_act = short_conv_silu(k_raw, P["k_conv_w"].to(wide))
        v_act = short_conv_silu(v_raw, P["v_conv_w"].to(wide))
    else:
        q_act, k_act, v_act = F.silu(q_raw), F.silu(k_raw), F.silu(v_raw)
    f_out = up((x @ P["f_proj_0"]) @ P["f_proj_1"])
    a = torch.exp(P["A_log"].to(wide)).repeat_interleave(hk)
    g = -a * F.softplus(f_out + P["dt_bias"].to(wide))  # src/module.rs:417-431
    if cfg.min_decay is not None:  # src/module.rs:432-440
        factor = torch.sigmoid(P["decay_factors"].to(wide)).reshape(kd) * (1.0 - cfg.min_decay)
        g = torch.log(factor * torch.exp(g) + cfg.min_decay)
    b = torch.sigmoid(up(x @ P["b_proj"]))
    w = torch.sigmoid(up(x @ P["w_proj"]))
    to4 = lambda t, n, d: t.reshape(B, T, n, d).permute(0, 2, 1, 3)
    q4, k4 = l2_normalize(to4(q_act, h, hk)), l2_normalize(to4(k_act, h, hk))
    g4, b4 = to4(g, h, hk), to4(b, h, hk)
    if hv > h:
        rep = hv // h
        q4, k4, g4, b4 = (gva_repeat(t, rep, gva_mode) for t in (q4, k4, g4, b4))
    if cfg.allow_neg_eigval:  # src/module.rs:470-472
        b4 = b4 * 2.0
    gate = up((x @ P["g_proj_0"]) @ P["g_proj_1_w"] + P["g_proj_1_b"]).reshape(B, T, hv, vh)
    cd = lambda t: t.to(core_dtype)
    return cd(q4), cd(k4), cd(to4(v_act, hv, vh)), g4.float() if wide == torch.float32 else g4, cd(b4), \
        cd(to4(w, hv, vh)), gate


def rms_norm_gate(o: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """o / sqrt(mean_V o^2 + eps) * weight * silu(gate) per head (src/module.rs:501-517); [B,T,HV,V]."""
    return o * torch.rsqrt((o * o).mean(-1, keepdim=True) + eps) * weight * F.silu(gate)


def cuda_core(q, k, v, g, b, w, scale, chunk):
    """The recurrence from a zero state on the B200 kernels: GatedDeltaCore."""
    return GatedDeltaCore.apply(q, k, v, g, b, w, None, scale, chunk)


def layer_forward(params: Dict[str, torch.Tensor], cfg: Gdn2Config, x: torch.Tensor, gva_mode: str = "reference",
                  core: Callable = cuda_core, core_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """forward_train (src/module.rs:326-375) as a torch autograd graph: x
    [B,T,D] -> [B,T,D]."""
    cfg.validate()
    h, hk, hv, vh = cfg.num_heads, cfg.head_dim, cfg.hv, cfg.v_head
    B, T, _ = x.shape
    cdt = core_dtype if core_dtype is not None else x.dtype
    q, k, v, g, b, w, gate = project(params, cfg, x, gva_mode, cdt)
    o, _ = core(q, k, v, g, b, w, hk ** -0.5, cfg.chunk_size)
    o4 = o.permute(0, 2, 1, 3).to(gate.dtype)  # [B,T,HV,V]
    normed = rms_norm_gate(o4, gate, params["o_norm_w"].to(gate.dtype), cfg.norm_eps)
    return normed.reshape(B, T, hv * vh).to(x.dtype) @ params["o_proj"]
