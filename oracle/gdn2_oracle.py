"""CPU oracle for the GDN-2 token-mixer hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``burn_gdn2`` over ``libgdn2_b200.so``) never
calls into this file and fails loudly when its CUDA library is missing.

It restates, in numpy, the algorithms of the reference crate
sehaxe/burn-gdn2 v0.5.1 (a Rust/burn crate that cannot be compiled here:
no cargo/rustc, burn 0.21 not vendored).  Every function cites the
reference file:line it follows.  The restatement is pinned against the
reference's own Python transcription ``tests/gen_reference.py`` through the
golden fixtures in ``tests/golden/`` (see ``tests/golden/gen_golden.py``).

All arithmetic runs in the dtype of the inputs (float64 for pinning,
float32 to mimic burn-ndarray's f32 tensor path).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import numpy as np

SHORT_CONV_KERNEL = 4  # src/short_conv.rs:5
SHORT_CONV_CACHE = 3  # src/short_conv.rs:7
FUSED_RECURRENT_MAX_SEQ = 64  # src/module.rs:17
TILE = 16  # src/forward.rs:90


# --------------------------------------------------------------------------
# elementwise helpers (burn activations)
# --------------------------------------------------------------------------
def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def silu(x):
    return x * sigmoid(x)


def softplus(x):
    # burn::tensor::activation::softplus(x, beta=1) = log(1 + exp(x))
    return np.logaddexp(0.0, x)


# --------------------------------------------------------------------------
# src/l2norm.rs:13-16
# --------------------------------------------------------------------------
def l2_normalize_4d(x, eps=1e-6):
    """x / sqrt(sum_K x^2 + eps) along the last dim (src/l2norm.rs:13-16)."""
    norm = np.sqrt((x * x).sum(axis=-1, keepdims=True) + x.dtype.type(eps))
    return x / norm


# --------------------------------------------------------------------------
# src/short_conv.rs:22-65
# --------------------------------------------------------------------------
def short_conv_1d(x, weight, cache=None):
    """Causal depthwise conv (kernel 4) + SiLU (src/short_conv.rs:22-65).

    x: [B,T,C]; weight: [C,4]; cache: [B,3,C] (oldest -> newest) or None.
    Without a cache the sequence start is padded by replicating x[:,0]
    three times (src/short_conv.rs:42-54).  Returns (silu(conv), new_cache)
    where new_cache = rows T..T+3 of the padded sequence (:30-55).
    """
    b, t, c = x.shape
    if cache is not None:
        x_pad = np.concatenate([cache, x], axis=1)
    else:
        x_pad = np.concatenate([np.repeat(x[:, :1], SHORT_CONV_CACHE, axis=1), x], axis=1)
    new_cache = x_pad[:, t:t + SHORT_CONV_CACHE].copy()
    out = np.zeros_like(x)
    for i in range(SHORT_CONV_KERNEL):
        out = out + x_pad[:, i:i + t] * weight[:, i].reshape(1, 1, c)
    return silu(out), new_cache


# --------------------------------------------------------------------------
# src/module.rs:501-517
# --------------------------------------------------------------------------
def rms_norm_gate_per_head(x, gate, weight, eps):
    """x / sqrt(mean_V x^2 + eps) * weight * silu(gate) (src/module.rs:501-517).

    x, gate: [B,T,HV,V]; weight: [V].
    """
    rms = np.sqrt((x * x).mean(axis=3, keepdims=True) + x.dtype.type(eps))
    return x / rms * weight.reshape(1, 1, 1, -1) * silu(gate)


# --------------------------------------------------------------------------
# src/kernel/fused_recurrent.rs:11-56
# --------------------------------------------------------------------------
def fused_recurrent_forward(q, k, v, g, b, w, state, scale):
    """Token-by-token scan (src/kernel/fused_recurrent.rs:11-56).

    q,k,g,b: [B,HV,T,K] (g and b may have last dim 1: broadcast);
    v,w: [B,HV,T,V]; state [B,HV,K,V].  Returns (out [B,HV,T,V], state).
    Per token:  S <- S*exp(g_t)            (:36)
                v_new = w*v - (b*k)^T S     (:39-41)
                S <- S + k v_new^T          (:44)
                o = scale * q^T S           (:47-49)
    """
    T = q.shape[2]
    S = state.copy()
    g_exp = np.exp(g)
    outs = []
    for t in range(T):
        S = S * g_exp[:, :, t, :, None]
        bk = (b[:, :, t] * k[:, :, t])[..., None]  # [B,H,K,1]
        erased = (S * bk).sum(axis=2)  # [B,H,V]
        v_new = w[:, :, t] * v[:, :, t] - erased
        S = S + k[:, :, t, :, None] * v_new[:, :, None, :]
        o = (S * q[:, :, t, :, None]).sum(axis=2) * scale
        outs.append(o)
    return np.stack(outs, axis=2), S


def fused_recurrent_trajectory(q, k, v, g, b, w, state, chunk):
    """What gdn2_chunk_trajectory_export_kernel (src/kernel/chunk_cube.rs:613-734)
    exports for a backward: the state entering every chunk of `chunk` tokens
    [B,H,ceil(T/chunk),K,V] and v_new [B,H,T,V].  The crate forms v_new of a
    chunk as u - w S (its WY factors); per token that is w v - (b k)^T (e^g S),
    the recurrence of src/kernel/fused_recurrent.rs:36-44, stepped here."""
    B, H, T, K = q.shape
    S = state.copy()
    gam = np.exp(g)
    states, vnew = [], np.zeros(v.shape, dtype=S.dtype)
    for t in range(T):
        if t % chunk == 0:
            states.append(S.copy())
        Sa = S * gam[:, :, t, :, None]
        bk = b[:, :, t] * k[:, :, t]
        u = w[:, :, t] * v[:, :, t] - (Sa * bk[..., None]).sum(axis=2)
        vnew[:, :, t] = u
        S = Sa + k[:, :, t, :, None] * u[:, :, None, :]
    return np.stack(states, axis=2), vnew


def fused_recurrent_backward(q, k, v, g, b, w, state, scale, d_out, d_state=None):
    """Reverse-mode adjoint of fused_recurrent_forward (the recurrence of
    src/kernel/fused_recurrent.rs:11-56, which the crate differentiates by
    burn autodiff of src/forward.rs:44-278).  Stores every token's state,
    then walks the tokens backwards.

    Shapes as fused_recurrent_forward with g, b of last dim K; d_out
    [B,H,T,V]; d_state dL/d(final state) or None.  Returns
    (dq, dk, dv, dg, db, dw, d_state_in).
    """
    T = q.shape[2]
    S = state.copy()
    gam = np.exp(g)
    pre = []  # the incoming state of every token
    us = []
    for t in range(T):
        pre.append(S)
        Sa = S * gam[:, :, t, :, None]
        bk = b[:, :, t] * k[:, :, t]
        u = w[:, :, t] * v[:, :, t] - (Sa * bk[..., None]).sum(axis=2)
        S = Sa + k[:, :, t, :, None] * u[:, :, None, :]
        us.append(u)
    dS = np.zeros_like(S) if d_state is None else d_state.astype(S.dtype).copy()
    dq, dk, dg, db = (np.zeros_like(q) for _ in range(4))
    dv, dw = np.zeros_like(v), np.zeros_like(w)
    for t in range(T - 1, -1, -1):
        gt = gam[:, :, t, :, None]
        kt, qt, bt = k[:, :, t], q[:, :, t], b[:, :, t]
        Sa = pre[t] * gt
        St = Sa + kt[..., None] * us[t][:, :, None, :]
        dO = d_out[:, :, t]
        dS = dS + scale * qt[..., None] * dO[:, :, None, :]  # o_t = scale S_t^T q_t
        dq[:, :, t] = scale * (St * dO[:, :, None, :]).sum(axis=3)
        du = (dS * kt[..., None]).sum(axis=2)  # S_t = Sa + k u^T
        dk[:, :, t] = (dS * us[t][:, :, None, :]).sum(axis=3)
        dv[:, :, t] = du * w[:, :, t]  # u = w v - e
        dw[:, :, t] = du * v[:, :, t]
        dSa = dS - (bt * kt)[..., None] * du[:, :, None, :]  # e = Sa^T (b k), de = -du
        dbk = -(Sa * du[:, :, None, :]).sum(axis=3)
        dk[:, :, t] += dbk * bt
        db[:, :, t] = dbk * kt
        dg[:, :, t] = (dSa * Sa).sum(axis=3)  # Sa = e^g S_{t-1}
        dS = dSa * gt
    return dq, dk, dv, dg, db, dw, dS


# --------------------------------------------------------------------------
# src/forward.rs:44-278
# --------------------------------------------------------------------------
def _pad_time(x, c_pad):
    """src/forward.rs:34-41 — zero-pad the time axis of a [B,H,c,d] chunk."""
    c = x.shape[2]
    if c == c_pad:
        return x
    pad = np.zeros(x.shape[:2] + (c_pad - c,) + x.shape[3:], dtype=x.dtype)
    return np.concatenate([x, pad], axis=2)


def chunk_wy_forward(q, k, v, g, b, w, state, scale, chunk_size):
    """Chunked WY forward with the tile-local log-space decay scheme.

    Restates src/forward.rs:44-278 step by step:
      * chunk loop, last chunk partial and zero-padded to a multiple of 16
        (:60-99);
      * G = inclusive cumsum of g per channel (:101-108), tile boundaries
        Gb (:109-129), tile-local E = exp(G - Gb) (:131-139), gamma = exp(G)
        (:141-142), inter-tile exp(min(Gb_p - Gb_q, 0)) (:144-157);
      * Aqk = scale * causal( sum_k (q E)(k / E)^T e_block ),
        Akk = strict( sum_k (b k E)(k / E)^T e_block ) (:159-187);
      * rhs_k = b k gamma, rhs_v = w v (:189-190);
      * (I + Akk) [W | U] = [rhs_k | rhs_v] by blocked forward substitution
        over 16-row tiles (:192-261);
      * v_new = U - W S; o = Aqk v_new + scale (q gamma) S (:263-269);
      * S <- diag(gamma_last) S + (k exp(G_last - G))^T v_new (:271-274).
    g and b may have last dim 1 (scalar broadcast over K, ``k % g_dim``).
    """
    B, H, T, K = q.shape
    V = v.shape[3]
    dt = q.dtype
    S = state.astype(dt, copy=True)
    outs = []
    for start in range(0, T, chunk_size):
        end = min(start + chunk_size, T)
        c = end - start
        if c == 0:
            continue
        c_pad = -(-c // TILE) * TILE
        n_t = c_pad // TILE
        qp = _pad_time(q[:, :, start:end], c_pad)
        kp = _pad_time(k[:, :, start:end], c_pad)
        vp = _pad_time(v[:, :, start:end], c_pad)
        gp = _pad_time(g[:, :, start:end], c_pad)
        bp = _pad_time(b[:, :, start:end], c_pad)
        wp = _pad_time(w[:, :, start:end], c_pad)
        gd = gp.shape[3]
        bd = bp.shape[3]

        G = np.cumsum(gp, axis=2)  # [B,H,c_pad,gd]
        Gb = np.zeros((B, H, n_t, gd), dtype=dt)
        if n_t > 1:
            Gb[:, :, 1:] = G[:, :, TILE - 1:c_pad - 1:TILE]
        Gb_full = np.repeat(Gb, TILE, axis=2)
        E = np.exp(G - Gb_full)
        gamma = np.exp(G)

        # per-channel inter-tile weight exp(min(Gb_p - Gb_q, 0)): [B,H,n_t,n_t,gd]
        eb = np.exp(np.minimum(Gb[:, :, :, None, :] - Gb[:, :, None, :, :], 0.0))
        kidx = np.arange(K)
        Eg = E[..., kidx % gd]  # [B,H,c_pad,K]
        ebk = eb[..., kidx % gd]  # [B,H,n_t,n_t,K]
        bk_full = bp[..., kidx % bd]
        qE = qp * Eg
        kE = kp / Eg
        bkE = bk_full * kp * Eg
        aqk = np.zeros((B, H, c_pad, c_pad), dtype=dt)
        akk = np.zeros((B, H, c_pad, c_pad), dtype=dt)
        for p in range(n_t):
            rp = slice(p * TILE, (p + 1) * TILE)
            for qq in range(n_t):
                rq = slice(qq * TILE, (qq + 1) * TILE)
                wgt = ebk[:, :, p, qq][:, :, None, :]  # [B,H,1,K]
                aqk[:, :, rp, rq] = np.einsum("bhrk,bhsk->bhrs", qE[:, :, rp] * wgt, kE[:, :, rq])
                akk[:, :, rp, rq] = np.einsum("bhrk,bhsk->bhrs", bkE[:, :, rp] * wgt, kE[:, :, rq])
        causal = np.tril(np.ones((c_pad, c_pad), dtype=dt))
        strict = np.tril(np.ones((c_pad, c_pad), dtype=dt), -1)
        aqk = aqk * dt.type(scale) * causal
        akk = akk * strict

        rhs_k = bp * kp * gamma
        rhs_v = wp * vp

        Wm = np.zeros((B, H, c_pad, K), dtype=dt)
        Um = np.zeros((B, H, c_pad, V), dtype=dt)
        for p in range(n_t):
            r0 = p * TILE
            t_pp = akk[:, :, r0:r0 + TILE, r0:r0 + TILE]
            wb = rhs_k[:, :, r0:r0 + TILE].copy()
            ub = rhs_v[:, :, r0:r0 + TILE].copy()
            if r0 > 0:
                t_pq = akk[:, :, r0:r0 + TILE, :r0]
                wb = wb - t_pq @ Wm[:, :, :r0]
                ub = ub - t_pq @ Um[:, :, :r0]
            for i in range(1, TILE):
                t_row = t_pp[:, :, i:i + 1, :i]
                wb[:, :, i:i + 1] = wb[:, :, i:i + 1] - t_row @ wb[:, :, :i]
                ub[:, :, i:i + 1] = ub[:, :, i:i + 1] - t_row @ ub[:, :, :i]
            Wm[:, :, r0:r0 + TILE] = wb
            Um[:, :, r0:r0 + TILE] = ub

        v_new = Um - Wm @ S
        intra = aqk @ v_new
        inter = (qp * gamma) @ S * dt.type(scale)
        outs.append((intra + inter)[:, :, :c])

        g_last = gamma[:, :, c - 1]  # [B,H,gd]
        g_last_log = G[:, :, c - 1:c]
        decay_last = np.exp(g_last_log - G)  # [B,H,c_pad,gd]
        S = S * g_last[:, :, :, None] + np.swapaxes(kp * decay_last, 2, 3) @ v_new
    return np.concatenate(outs, axis=2), S


# --------------------------------------------------------------------------
# src/config.rs
# --------------------------------------------------------------------------
@dataclasses.dataclass
class Gdn2Config:
    """Mirror of ``Gdn2Config`` (src/config.rs:24-58, defaults :114-129)."""

    hidden_size: int = 2048
    num_heads: int = 16
    head_dim: int = 128
    expand_v: float = 1.0
    num_v_heads: Optional[int] = None
    use_short_conv: bool = True
    allow_neg_eigval: bool = False
    norm_eps: float = 1e-5
    mode: str = "fused_recurrent"  # or "chunk"
    chunk_size: int = 64
    min_decay: Optional[float] = None

    def validate(self):
        """Panicking checks of src/config.rs:71-111, raised as ValueError."""
        h, hk = self.num_heads, self.head_dim
        if self.hidden_size <= 0:
            raise ValueError(f"hidden_size must be > 0, got {self.hidden_size}")
        if h <= 0:
            raise ValueError(f"num_heads must be > 0, got {h}")
        if hk <= 0:
            raise ValueError(f"head_dim must be > 0, got {hk}")
        prod = np.float32(hk) * np.float32(self.expand_v)
        if not (self.expand_v > 0.0 and float(prod) == math.floor(float(prod))):
            raise ValueError(f"expand_v={self.expand_v} must produce an integer head_v_dim")
        if self.num_v_heads is not None:
            hv = self.num_v_heads
            if hv <= 0:
                raise ValueError(f"num_v_heads must be > 0, got {hv}")
            if hv < h:
                raise ValueError(f"num_v_heads={hv} < num_heads={h} is not supported")
            if hv % h != 0:
                raise ValueError(f"num_v_heads={hv} must be divisible by num_heads={h}")
        if self.chunk_size <= 0:
            raise ValueError(f"chunk_size must be > 0, got {self.chunk_size}")
        if not self.norm_eps > 0.0:
            raise ValueError(f"norm_eps must be > 0, got {self.norm_eps}")

    @property
    def hv(self):
        return self.num_v_heads if self.num_v_heads is not None else self.num_heads

    @property
    def v_head(self):
        return int(np.float32(self.head_dim) * np.float32(self.expand_v))


# --------------------------------------------------------------------------
# src/module.rs:111-189 (weights), seeded re-sampling of the same laws
# --------------------------------------------------------------------------
def init_weights(cfg: Gdn2Config, seed: int = 0, dtype=np.float32):
    """Random-init weights with the distributions of src/module.rs:111-189.

    burn's RNG stream cannot be reproduced without burn, so the same laws are
    re-sampled from a seeded numpy generator:
      Linear: Xavier-uniform, gain 2^-2.5, stored [in, out] (burn layout);
      g_proj_1 bias 0; conv weights U(-0.5, 0.5) [C, 4];
      A_log = U(ln 1, ln 16) [H]; dt = exp(U(ln 1e-3, ln 0.1)) clamped >= 1e-4,
      dt_bias = dt + ln(1 - exp(-dt)); o_norm = 1 [V]; decay_factors = 2 [H, K].
    """
    cfg.validate()
    rng = np.random.default_rng(seed)
    d, h, hk = cfg.hidden_size, cfg.num_heads, cfg.head_dim
    hv, vh = cfg.hv, cfg.v_head
    kd, vd = h * hk, hv * vh
    gain = 2.0 ** -2.5

    def lin(i, o):
        a = gain * math.sqrt(6.0 / (i + o))
        return rng.uniform(-a, a, size=(i, o)).astype(dtype)

    wts = {
        "q_proj": lin(d, kd),
        "k_proj": lin(d, kd),
        "v_proj": lin(d, vd),
        "f_proj_0": lin(d, vh),
        "f_proj_1": lin(vh, kd),
        "b_proj": lin(d, kd),
        "w_proj": lin(d, vd),
        "g_proj_0": lin(d, vh),
        "g_proj_1_w": lin(vh, vd),
        "g_proj_1_b": np.zeros(vd, dtype=dtype),
        "A_log": rng.uniform(math.log(1.0), math.log(16.0), size=h).astype(dtype),
    }
    dt = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=kd))
    dt = np.maximum(dt, 1e-4)
    wts["dt_bias"] = (dt + np.log(-np.expm1(-dt))).astype(dtype)
    wts["o_norm_w"] = np.ones(vh, dtype=dtype)
    wts["o_proj"] = lin(vd, d)
    wts["q_conv_w"] = rng.uniform(-0.5, 0.5, size=(kd, 4)).astype(dtype)
    wts["k_conv_w"] = rng.uniform(-0.5, 0.5, size=(kd, 4)).astype(dtype)
    wts["v_conv_w"] = rng.uniform(-0.5, 0.5, size=(vd, 4)).astype(dtype)
    if cfg.min_decay is not None:
        wts["decay_factors"] = np.full((h, hk), 2.0, dtype=dtype)
    return wts


@dataclasses.dataclass
class Gdn2State:
    """Mirror of ``Gdn2State`` (src/module.rs:31-64)."""

    recurrent: np.ndarray  # [B,HV,K,V]
    conv_q: np.ndarray  # [B,3,H*K]
    conv_k: np.ndarray  # [B,3,H*K]
    conv_v: np.ndarray  # [B,3,HV*V]


def gva_repeat_ref(x, rep):
    """GVA repeat of src/module.rs:457-468, reproduced exactly.

    ``unsqueeze(3).repeat([1,1,1,rep,1]).reshape([B,HV,T,K])``: value head
    ``h*rep + j`` at time ``t`` reads key-side token ``(j*T + t) // rep``.
    For T == 1 this equals the plain head repeat.
    """
    B, H, T, K = x.shape
    return np.repeat(x[:, :, :, None, :], rep, axis=3).reshape(B, H * rep, T, K)


class Gdn2Layer:
    """Numpy restatement of ``GatedDeltaNet2`` (src/module.rs:83-498)."""

    def __init__(self, cfg: Gdn2Config, weights: dict, dtype=np.float64, gva="reference"):
        """gva="reference" reproduces src/module.rs:457-468 exactly;
        gva="grouped" gives value head hv key head hv // rep at the same
        token (the product's optional corrected mode, equal for T == 1)."""
        cfg.validate()
        self.cfg = cfg
        self.gva = gva
        self.dtype = dtype
        self.w = {k: np.asarray(v, dtype=dtype) for k, v in weights.items()}

    # src/module.rs:381-498
    def project(self, x, conv_cache=None):
        cfg, W = self.cfg, self.w
        x = np.asarray(x, dtype=self.dtype)
        B, T, _ = x.shape
        h, hk, hv, vh = cfg.num_heads, cfg.head_dim, cfg.hv, cfg.v_head
        kd, vd = h * hk, hv * vh

        def to_4d(t, n, d):
            return t.reshape(B, T, n, d).transpose(0, 2, 1, 3)

        q_raw = x @ W["q_proj"]
        k_raw = x @ W["k_proj"]
        v_raw = x @ W["v_proj"]
        if cfg.use_short_conv:
            cq, ck, cv = conv_cache if conv_cache is not None else (None, None, None)
            q_act, nq = short_conv_1d(q_raw, W["q_conv_w"], cq)
            k_act, nk = short_conv_1d(k_raw, W["k_conv_w"], ck)
            v_act, nv = short_conv_1d(v_raw, W["v_conv_w"], cv)
            conv_out = (nq, nk, nv)
        else:
            q_act, k_act, v_act = silu(q_raw), silu(k_raw), silu(v_raw)
            conv_out = None

        f_out = (x @ W["f_proj_0"]) @ W["f_proj_1"]
        a_exp = np.repeat(np.exp(W["A_log"]), hk).reshape(1, 1, kd)
        g = -a_exp * softplus(f_out + W["dt_bias"].reshape(1, 1, kd))
        if cfg.min_decay is not None:
            alpha = 1.0 - cfg.min_decay
            factor = (sigmoid(W["decay_factors"]) * alpha).reshape(1, 1, kd)
            g = np.log(factor * np.exp(g) + cfg.min_decay)

        b_gate = sigmoid(x @ W["b_proj"])
        w_gate = sigmoid(x @ W["w_proj"])

        q4 = l2_normalize_4d(to_4d(q_act, h, hk), 1e-6)
        k4 = l2_normalize_4d(to_4d(k_act, h, hk), 1e-6)
        v4 = to_4d(v_act, hv, vh)
        g4 = to_4d(g, h, hk)
        b4 = to_4d(b_gate, h, hk)
        w4 = to_4d(w_gate, hv, vh)
        if hv > h:
            rep = hv // h
            rep_fn = gva_repeat_ref if self.gva == "reference" else (lambda t, r: np.repeat(t, r, axis=1))
            q4, k4, g4, b4 = (rep_fn(t, rep) for t in (q4, k4, g4, b4))
        if cfg.allow_neg_eigval:
            b4 = b4 * 2.0
        gate = ((x @ W["g_proj_0"]) @ W["g_proj_1_w"] + W["g_proj_1_b"]).reshape(B, T, hv, vh)
        proj = dict(q=q4, k=k4, v=v4, g=g4, b=b4, w=w4, gate=gate)
        return proj, conv_out

    def _epilogue(self, o_bhtv, gate):
        B, HV, T, V = o_bhtv.shape
        o4 = o_bhtv.transpose(0, 2, 1, 3)
        normed = rms_norm_gate_per_head(o4, gate, self.w["o_norm_w"], self.cfg.norm_eps)
        return normed.reshape(B, T, HV * V) @ self.w["o_proj"]

    # src/module.rs:224-316
    def forward(self, x, state: Optional[Gdn2State] = None, update_state=True):
        """Returns (y [B,T,D], state).  ``state`` None = fresh sequence."""
        cfg = self.cfg
        B, T, _ = x.shape
        hk, hv, vh = cfg.head_dim, cfg.hv, cfg.v_head
        conv_in = (state.conv_q, state.conv_k, state.conv_v) if state is not None else None
        p, conv_out = self.project(x, conv_in)
        scale = hk ** -0.5
        rec = state.recurrent if state is not None else np.zeros((B, hv, hk, vh), dtype=self.dtype)
        if update_state:
            mode = "fused_recurrent" if T <= FUSED_RECURRENT_MAX_SEQ else cfg.mode
            if mode == "fused_recurrent":
                o, new_rec = fused_recurrent_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], rec, scale)
            else:
                o, new_rec = chunk_wy_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], rec, scale,
                                              cfg.chunk_size)
            kd, vd = cfg.num_heads * hk, hv * vh
            if state is None:
                z = np.zeros
                state = Gdn2State(z((B, hv, hk, vh), self.dtype), z((B, 3, kd), self.dtype),
                                  z((B, 3, kd), self.dtype), z((B, 3, vd), self.dtype))
            state.recurrent = new_rec
            if conv_out is not None:
                state.conv_q, state.conv_k, state.conv_v = conv_out
        else:
            # read-only: o_t = scale * q_t^T S (state untouched), the evident intent
            # of src/module.rs:297-308, whose output is permuted twice (:307, :310).
            o = p["q"] @ rec * scale
        return self._epilogue(o, p["gate"]), state

    # src/module.rs:326-375
    def forward_train(self, x):
        cfg = self.cfg
        B, T, _ = x.shape
        hk, hv, vh = cfg.head_dim, cfg.hv, cfg.v_head
        p, _ = self.project(x, None)
        scale = hk ** -0.5
        S0 = np.zeros((B, hv, hk, vh), dtype=self.dtype)
        if cfg.mode == "fused_recurrent":
            o, _ = fused_recurrent_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], S0, scale)
        else:
            o, _ = chunk_wy_forward(p["q"], p["k"], p["v"], p["g"], p["b"], p["w"], S0, scale, cfg.chunk_size)
        return self._epilogue(o, p["gate"])


# --------------------------------------------------------------------------
# seeded synthetic core inputs (shapes of BASELINE.json configs)
# --------------------------------------------------------------------------
def make_core_inputs(B, HV, T, K, V, seed=0, decay=(-0.15, -0.01), dtype=np.float32, neg_eig=False):
    """Seeded inputs for the core kernels with the value laws the module
    produces: q,k L2-normalised (src/module.rs:453-454), g < 0 per channel,
    b, w in (0,1) (sigmoid gates, b in (0,2) with neg-eig), v ~ N(0,1),
    gate ~ N(0,1) [B,T,HV,V]."""
    rng = np.random.default_rng(seed)
    q = l2_normalize_4d(rng.standard_normal((B, HV, T, K)), 1e-6)
    k = l2_normalize_4d(rng.standard_normal((B, HV, T, K)), 1e-6)
    v = rng.standard_normal((B, HV, T, V))
    g = rng.uniform(decay[0], decay[1], size=(B, HV, T, K))
    b = rng.uniform(0.0, 1.0, size=(B, HV, T, K)) * (2.0 if neg_eig else 1.0)
    w = rng.uniform(0.0, 1.0, size=(B, HV, T, V))
    gate = rng.standard_normal((B, T, HV, V))
    out = dict(q=q, k=k, v=v, g=g, b=b, w=w, gate=gate)
    return {n: a.astype(dtype) for n, a in out.items()}
