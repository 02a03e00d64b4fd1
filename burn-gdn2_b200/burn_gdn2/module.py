"""GatedDeltaNet2 / Gdn2State — mirror of src/module.rs (sehaxe/burn-gdn2 v0.5.1).

The projections (burn ``Linear``, weights stored ``[in, out]``) are cuBLAS
GEMMs through torch; everything recurrent runs in libgdn2_b200.so:

* ``forward`` with T <= 64 tokens (or mode FusedRecurrent) -> kernel (3),
  with the short conv + SiLU + L2 prologue and the gated RMS-norm epilogue
  fused into the same launch, state and conv caches updated in place;
* longer sequences in mode Chunk and ``forward_train`` in mode Chunk ->
  kernels (1) + (2) with the fused epilogue.

GVA (num_v_heads > num_heads): the reference repeats key-side tensors with
``unsqueeze(3).repeat(..).reshape`` (src/module.rs:457-468), which for T > 1
hands value head ``h*rep + j`` the key-side tokens ``(j*T + t) // rep``.
``gva_mode="reference"`` (default) reproduces that exactly;
``gva_mode="grouped"`` gives value head ``hv`` key head ``hv // rep`` at the
same token (identical for T == 1) without materialising the repeat.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math
from typing import Optional

import torch

from . import _lib
from ._lib import LIB, check
from .config import Gdn2Config, Gdn2Mode
from .ops import (SHORT_CONV_CACHE, chunk_args, chunk_workspace, precision_code, project_activations,
                  recurrent_args, rms_norm_gate_per_head, stream_handle)

FUSED_RECURRENT_MAX_SEQ = 64  # src/module.rs:17


@dataclasses.dataclass
class Linear:
    """burn Linear: y = x W (+ b), W stored [in, out]."""

    weight: torch.Tensor
    bias: Optional[torch.Tensor] = None

    def forward(self, x):
        y = x @ self.weight
        return y if self.bias is None else y + self.bias


@dataclasses.dataclass
class Gdn2State:
    """Recurrent + short-conv state (src/module.rs:31-64).

    recurrent [B,HV,K,V] f32; conv_q, conv_k [B,3,H*K] f32; conv_v [B,3,HV*V]
    f32 (oldest -> newest).  Updated in place by ``forward``.
    """

    recurrent: torch.Tensor
    conv_q: torch.Tensor
    conv_k: torch.Tensor
    conv_v: torch.Tensor

    @staticmethod
    def zeros(device, batch, hv, hk, v_head, kd, vd):
        z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=device)
        return Gdn2State(z(batch, hv, hk, v_head), z(batch, SHORT_CONV_CACHE, kd), z(batch, SHORT_CONV_CACHE, kd),
                         z(batch, SHORT_CONV_CACHE, vd))


@dataclasses.dataclass
class ProjectedInputs:
    """src/module.rs:519-532."""

    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    g: torch.Tensor
    b: torch.Tensor
    w: torch.Tensor
    gate: torch.Tensor
    o_norm: torch.Tensor
    eps: float
    hv: int
    vd: int
    grouped: bool = False


class GatedDeltaNet2:
    """GDN-2 token-mixing layer (src/module.rs:83-498)."""

    NAMES = ("q_proj", "k_proj", "v_proj", "f_proj_0", "f_proj_1", "b_proj", "w_proj", "g_proj_0", "g_proj_1_w",
             "g_proj_1_b", "A_log", "dt_bias", "o_norm_w", "o_proj", "q_conv_w", "k_conv_w", "v_conv_w")

    def __init__(self, cfg: Gdn2Config, weights: dict, device="cuda", dtype=torch.float32, gva_mode="reference",
                 precision="f32"):
        cfg.validate()
        if gva_mode not in ("reference", "grouped"):
            raise ValueError("gva_mode must be 'reference' or 'grouped'")
        precision_code(precision)
        self.precision = precision
        self.config = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.gva_mode = gva_mode
        W = {k: torch.as_tensor(v) for k, v in weights.items()}
        lin = lambda n: Linear(W[n].to(self.device, dtype))
        self.q_proj, self.k_proj, self.v_proj = lin("q_proj"), lin("k_proj"), lin("v_proj")
        self.f_proj_0, self.f_proj_1 = lin("f_proj_0"), lin("f_proj_1")
        self.b_proj, self.w_proj = lin("b_proj"), lin("w_proj")
        self.g_proj_0 = lin("g_proj_0")
        self.g_proj_1 = Linear(W["g_proj_1_w"].to(self.device, dtype), W["g_proj_1_b"].to(self.device, dtype))
        self.o_proj = lin("o_proj")
        f32 = lambda n: W[n].to(self.device, torch.float32).contiguous()
        self.a_log, self.dt_bias, self.o_norm_weight = f32("A_log"), f32("dt_bias"), f32("o_norm_w")
        self.q_conv_w, self.k_conv_w, self.v_conv_w = f32("q_conv_w"), f32("k_conv_w"), f32("v_conv_w")
        self.decay_factors = f32("decay_factors") if cfg.min_decay is not None else None

    # -- construction (src/module.rs:111-189) ------------------------------
    @classmethod
    def new(cls, cfg: Gdn2Config, device="cuda", dtype=torch.float32, seed=0, **kw):
        """Random init with the laws of src/module.rs:111-189 (seeded torch
        generator; burn's own RNG stream is not reproducible outside burn):
        Xavier-uniform gain 2^-2.5, zero g_proj_1 bias, conv U(-0.5, 0.5),
        A_log U(ln 1, ln 16), dt_bias = inverse-softplus of
        exp(U(ln 1e-3, ln 0.1)) >= 1e-4, o_norm = 1, decay_factors = 2."""
        cfg.validate()
        gen = torch.Generator().manual_seed(seed)
        d, h, hk, hv, vh = cfg.hidden_size, cfg.num_heads, cfg.head_dim, cfg.hv, cfg.v_head
        kd, vd = h * hk, hv * vh
        gain = 2.0 ** -2.5

        def lin(i, o):
            a = gain * math.sqrt(6.0 / (i + o))
            return (torch.rand(i, o, generator=gen, dtype=torch.float64) * 2 - 1) * a

        def uni(lo, hi, *s):
            return torch.rand(*s, generator=gen, dtype=torch.float64) * (hi - lo) + lo

        W = {"q_proj": lin(d, kd), "k_proj": lin(d, kd), "v_proj": lin(d, vd), "f_proj_0": lin(d, vh),
             "f_proj_1": lin(vh, kd), "b_proj": lin(d, kd), "w_proj": lin(d, vd), "g_proj_0": lin(d, vh),
             "g_proj_1_w": lin(vh, vd), "g_proj_1_b": torch.zeros(vd, dtype=torch.float64),
             "A_log": uni(math.log(1.0), math.log(16.0), h)}
        dt = torch.exp(uni(math.log(1e-3), math.log(0.1), kd)).clamp(min=1e-4)
        W["dt_bias"] = dt + torch.log(-torch.expm1(-dt))
        W["o_norm_w"] = torch.ones(vh, dtype=torch.float64)
        W["o_proj"] = lin(vd, d)
        W["q_conv_w"] = uni(-0.5, 0.5, kd, 4)
        W["k_conv_w"] = uni(-0.5, 0.5, kd, 4)
        W["v_conv_w"] = uni(-0.5, 0.5, vd, 4)
        if cfg.min_decay is not None:
            W["decay_factors"] = torch.full((h, hk), 2.0, dtype=torch.float64)
        return cls(cfg, {k: v.float() for k, v in W.items()}, device=device, dtype=dtype, **kw)

    def export_weights(self) -> dict:
        """The layer's weights as the constructor takes them (names of
        WEIGHTS, projections [in, out]), f32 on the host: e.g. to build
        per-rank shards of this layer (sharding.shard_weights)."""
        f = lambda t: t.detach().float().cpu()
        W = {n: f(getattr(self, n).weight) for n in
             ("q_proj", "k_proj", "v_proj", "f_proj_0", "f_proj_1", "b_proj", "w_proj", "g_proj_0", "o_proj")}
        W["g_proj_1_w"], W["g_proj_1_b"] = f(self.g_proj_1.weight), f(self.g_proj_1.bias)
        for n, a in (("A_log", "a_log"), ("dt_bias", "dt_bias"), ("o_norm_w", "o_norm_weight"),
                     ("q_conv_w", "q_conv_w"), ("k_conv_w", "k_conv_w"), ("v_conv_w", "v_conv_w")):
            W[n] = f(getattr(self, a))
        if self.decay_factors is not None:
            W["decay_factors"] = f(self.decay_factors)
        return W

    # -- training (torch autograd; src/module.rs:326-375 under burn autodiff) --
    def parameters(self) -> dict:
        """The layer's live weight tensors by constructor name (projections
        [in, out]); set ``requires_grad`` on them (``requires_grad_``) and call
        ``forward_train_autograd`` to train."""
        P = {n: getattr(self, n).weight for n in
             ("q_proj", "k_proj", "v_proj", "f_proj_0", "f_proj_1", "b_proj", "w_proj", "g_proj_0", "o_proj")}
        P["g_proj_1_w"], P["g_proj_1_b"] = self.g_proj_1.weight, self.g_proj_1.bias
        for n, a in (("A_log", "a_log"), ("dt_bias", "dt_bias"), ("o_norm_w", "o_norm_weight"),
                     ("q_conv_w", "q_conv_w"), ("k_conv_w", "k_conv_w"), ("v_conv_w", "v_conv_w")):
            P[n] = getattr(self, a)
        if self.decay_factors is not None:
            P["decay_factors"] = self.decay_factors
        return P

    def requires_grad_(self, flag: bool = True):
        for t in self.parameters().values():
            t.requires_grad_(flag)
        return self

    def forward_train_autograd(self, hidden_states):
        """forward_train as a torch autograd graph (burn_gdn2.training): the
        same output as ``forward_train``, with gradients for every weight
        whose ``requires_grad`` is set and for the input.  The recurrence runs
        on the chunked kernels forward and gdn2_recurrent_bwd backward."""
        from .training import layer_forward

        self._validate_input(hidden_states)
        return layer_forward(self.parameters(), self.config, hidden_states.to(self.dtype), self.gva_mode)

    # -- helpers -------------------------------------------------------------
    @property
    def _dims(self):
        c = self.config
        return c.num_heads, c.head_dim, c.hv, c.v_head

    def _validate_input(self, x):
        if x.shape[-1] != self.config.hidden_size:
            raise ValueError(f"GatedDeltaNet2: expected hidden_states with last dim {self.config.hidden_size} "
                             f"but got {x.shape[-1]}. Check that the model hidden_size matches your input.")
        if not x.is_cuda:
            raise RuntimeError("GatedDeltaNet2 runs on the B200 CUDA kernels only; got a CPU tensor")

    # -- src/module.rs:381-498 ----------------------------------------------
    def _proj_weight(self):
        """[D, 3*KD + 2*VD + 2*vh] concatenation of the q, k, v, b, w,
        f_proj_0 and g_proj_0 weights: one GEMM reads x once.  Rebuilt when
        any of the weights is replaced or modified in place."""
        parts = (self.q_proj, self.k_proj, self.v_proj, self.b_proj, self.w_proj, self.f_proj_0, self.g_proj_0)
        key = tuple((l.weight.data_ptr(), l.weight._version) for l in parts)
        if getattr(self, "_wcat_key", None) != key:
            self._wcat = torch.cat([l.weight for l in parts], dim=1).contiguous()
            self._wcat_key = key
        return self._wcat

    def _projections(self, x):
        """The layer's GEMMs before the core: one GEMM of x against the
        concatenated q, k, v, b, w, f_proj_0 and g_proj_0 weights, then the
        f_proj_1 / g_proj_1 up-projections.  Returns the raw [B*T, C] column
        slices (q, k, v, b, w, f) of that output and the gate [B*T, VD]."""
        h, hk, hv, vh = self._dims
        B, T, _ = x.shape
        kd, vd = h * hk, hv * vh
        y = x.to(self.dtype).reshape(B * T, -1) @ self._proj_weight()
        o = [0, kd, 2 * kd, 2 * kd + vd, 3 * kd + vd, 3 * kd + 2 * vd, 3 * kd + 2 * vd + vh]
        cols = lambda i, n: y[:, o[i]:o[i] + n]
        f_raw = cols(5, vh) @ self.f_proj_1.weight
        gate = torch.addmm(self.g_proj_1.bias, cols(6, vh), self.g_proj_1.weight)
        return (cols(0, kd), cols(1, kd), cols(2, vd), cols(3, kd), cols(4, vd), f_raw), gate

    def project(self, x, conv_cache=None, grouped=None):
        """Projection pipeline.  Returns (ProjectedInputs, conv_out or None).
        q,k,g,b are [B,HV,T,K] views (or [B,H,T,K] with grouped=True).

        One GEMM for the q, k, v, b, w and low-rank f / gate projections,
        the two low-rank up-projections, then gdn2_project_activations for
        every elementwise step (short conv, SiLU, L2, sigmoid gates, decay)."""
        self._validate_input(x)
        c = self.config
        h, hk, hv, vh = self._dims
        B, T, _ = x.shape
        kd, vd = h * hk, hv * vh
        grouped = (self.gva_mode == "grouped") if grouped is None else grouped
        raws, gate = self._projections(x)
        conv_w = (self.q_conv_w, self.k_conv_w, self.v_conv_w) if c.use_short_conv else None
        (q, k, v, b, w, g), conv_out = project_activations(
            *raws, batch=B, num_heads=h,
            head_k_dim=hk, num_v_heads=hv, head_v_dim=vh, a_log=self.a_log, dt_bias=self.dt_bias, conv_w=conv_w,
            conv_in=conv_cache if c.use_short_conv else None, allow_neg_eigval=c.allow_neg_eigval,
            min_decay=c.min_decay, decay_factors=self.decay_factors)
        to4 = lambda t, n, d: t.reshape(B, T, n, d).permute(0, 2, 1, 3)
        q4, k4, g4, b4 = to4(q, h, hk), to4(k, h, hk), to4(g, h, hk), to4(b, h, hk)
        if hv > h and not grouped:
            rep = hv // h
            r = lambda t: t.unsqueeze(3).repeat(1, 1, 1, rep, 1).reshape(B, hv, T, hk)
            q4, k4, g4, b4 = r(q4), r(k4), r(g4), r(b4)
        p = ProjectedInputs(q=q4, k=k4, v=to4(v, hv, vh), g=g4, b=b4, w=to4(w, hv, vh),
                            gate=gate.reshape(B, T, hv, vh), o_norm=self.o_norm_weight, eps=c.norm_eps, hv=hv,
                            vd=vd, grouped=bool(grouped and hv > h))
        return p, conv_out

    # -- cores ----------------------------------------------------------------
    def _chunk_core(self, p: ProjectedInputs, state: torch.Tensor) -> torch.Tensor:
        """Kernels (1)+(2) with the fused epilogue; state updated in place.
        Returns the normed output [B,T,HV,V]."""
        h = self.config.num_heads
        B, _, T, K = p.q.shape
        hv, V = p.hv, p.v.shape[3]
        out = torch.empty(B, T, hv, V, dtype=p.v.dtype, device=p.v.device)
        a = chunk_args(p.q, p.k, p.v, p.g, p.b, p.w, state, out.permute(0, 2, 1, 3), K ** -0.5,
                       self.config.chunk_size, num_heads=h, grouped=p.grouped, gate=p.gate.permute(0, 2, 1, 3),
                       o_norm_weight=p.o_norm, norm_eps=p.eps, precision=self.precision)
        ws = chunk_workspace(a, p.v.device)
        check(LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                 stream_handle(p.v.device)))
        return out

    def _recurrent_fused(self, x, state: Optional[Gdn2State], recurrent: torch.Tensor):
        """Kernel (3) straight from the raw projections: short conv + SiLU +
        L2 prologue and gated RMS-norm epilogue in the same launch.
        Returns (normed [B,T,HV,V], conv_out triple)."""
        c = self.config
        h, hk, hv, vh = self._dims
        B, T, _ = x.shape
        raws, gate = self._projections(x)
        q_raw, k_raw, v_raw = raws[:3]  # convolved in the recurrent kernel's own prologue
        # b, w, g from the activations pass (its q/k/v outputs, SiLU only, are not used here)
        (_, _, _, b, w, g), _ = project_activations(
            *raws, batch=B, num_heads=h, head_k_dim=hk, num_v_heads=hv, head_v_dim=vh, a_log=self.a_log,
            dt_bias=self.dt_bias, conv_w=None, allow_neg_eigval=c.allow_neg_eigval, min_decay=c.min_decay,
            decay_factors=self.decay_factors)
        to4 = lambda t, n, d: t.reshape(B, T, n, d).permute(0, 2, 1, 3)
        kd, vd = h * hk, hv * vh
        if c.use_short_conv:
            cin = (state.conv_q, state.conv_k, state.conv_v) if state is not None else (None, None, None)
            if state is not None:
                cout = cin  # updated in place
            else:
                cout = tuple(torch.empty(B, SHORT_CONV_CACHE, n, dtype=torch.float32, device=x.device)
                             for n in (kd, kd, vd))
            conv_w = (self.q_conv_w, self.k_conv_w, self.v_conv_w)
            prologue = 1
        else:
            cin = cout = conv_w = (None, None, None)
            prologue = 2
        out = torch.empty(B, T, hv, vh, dtype=self.dtype, device=x.device)
        a = recurrent_args(to4(q_raw, h, hk), to4(k_raw, h, hk), to4(v_raw, hv, vh), to4(g, h, hk), to4(b, h, hk),
                           to4(w, hv, vh), recurrent, out.permute(0, 2, 1, 3), hk ** -0.5, num_heads=h,
                           grouped=True, prologue=prologue, conv_w=conv_w, conv_in=cin, conv_out=cout,
                           gate=to4(gate, hv, vh), o_norm_weight=self.o_norm_weight, norm_eps=c.norm_eps)
        st = LIB.gdn2_recurrent_fwd(ctypes.byref(a), stream_handle(x.device))
        if st == _lib.GDN2_EUNSUPPORTED and state is not None and c.use_short_conv:
            # too many CTAs share a cache for an in-place update: write fresh caches
            cout = tuple(torch.empty_like(t) for t in cin)
            a = recurrent_args(to4(q_raw, h, hk), to4(k_raw, h, hk), to4(v_raw, hv, vh), to4(g, h, hk),
                               to4(b, h, hk), to4(w, hv, vh), recurrent, out.permute(0, 2, 1, 3), hk ** -0.5,
                               num_heads=h, grouped=True, prologue=prologue, conv_w=conv_w, conv_in=cin,
                               conv_out=cout, gate=to4(gate, hv, vh), o_norm_weight=self.o_norm_weight,
                               norm_eps=c.norm_eps)
            st = LIB.gdn2_recurrent_fwd(ctypes.byref(a), stream_handle(x.device))
        check(st)
        return out, (cout if c.use_short_conv else None)

    def _recurrent_projected(self, p: ProjectedInputs, recurrent: torch.Tensor):
        """Kernel (3) on projected inputs (GVA reference layout), then the
        epilogue kernel.  Returns normed [B,T,HV,V]."""
        B, _, T, K = p.q.shape
        o = torch.empty(B, T, p.hv, p.v.shape[3], dtype=p.v.dtype, device=p.v.device)
        a = recurrent_args(p.q, p.k, p.v, p.g, p.b, p.w, recurrent, o.permute(0, 2, 1, 3), K ** -0.5,
                           num_heads=self.config.num_heads, grouped=p.grouped)
        check(LIB.gdn2_recurrent_fwd(ctypes.byref(a), stream_handle(p.v.device)))
        return rms_norm_gate_per_head(o, p.gate, p.o_norm, p.eps)

    def _out_proj(self, normed):
        B, T, hv, vh = normed.shape
        return self.o_proj.forward(normed.reshape(B, T, hv * vh))

    # -- src/module.rs:224-316 ------------------------------------------------
    def forward(self, hidden_states, state: Optional[Gdn2State] = None, update_state: bool = True):
        """Inference forward with state.  Returns (output [B,T,D], state).

        Mirrors ``forward(x, &mut Option<Gdn2State>, update_state)``: pass the
        previous state (or None for a fresh sequence); the returned state is
        the same object updated in place (or a new one when None was given).
        T <= 64 tokens always run the fused-recurrent kernel; longer inputs
        follow ``config.mode``."""
        self._validate_input(hidden_states)
        c = self.config
        h, hk, hv, vh = self._dims
        B, T, _ = hidden_states.shape
        kd, vd = h * hk, hv * vh
        dev = hidden_states.device
        if not update_state:
            conv_in = (state.conv_q, state.conv_k, state.conv_v) if state is not None else None
            p, _ = self.project(hidden_states, conv_in, grouped=False)
            mem = state.recurrent if state is not None else torch.zeros(B, hv, hk, vh, device=dev)
            o = (p.q.float() @ mem * hk ** -0.5).permute(0, 2, 1, 3).to(p.v.dtype)
            return self._out_proj(rms_norm_gate_per_head(o, p.gate, p.o_norm, p.eps)), state
        mode = Gdn2Mode.FusedRecurrent if T <= FUSED_RECURRENT_MAX_SEQ else Gdn2Mode(c.mode)
        recurrent = (state.recurrent if state is not None
                     else torch.zeros(B, hv, hk, vh, dtype=torch.float32, device=dev))
        conv_out = None
        if mode == Gdn2Mode.FusedRecurrent and (hv == h or T == 1 or self.gva_mode == "grouped"):
            normed, conv_out = self._recurrent_fused(hidden_states, state, recurrent)
        else:
            conv_in = (state.conv_q, state.conv_k, state.conv_v) if state is not None else None
            p, conv_out = self.project(hidden_states, conv_in)
            if mode == Gdn2Mode.FusedRecurrent:
                normed = self._recurrent_projected(p, recurrent)
            else:
                normed = self._chunk_core(p, recurrent)
        if state is None:
            state = Gdn2State.zeros(dev, B, hv, hk, vh, kd, vd)
            state.recurrent = recurrent
        if conv_out is not None:
            state.conv_q, state.conv_k, state.conv_v = conv_out
        return self._out_proj(normed), state

    # -- src/module.rs:326-375 ------------------------------------------------
    def forward_train(self, hidden_states):
        """Full-sequence forward from a zero state (no state returned)."""
        self._validate_input(hidden_states)
        h, hk, hv, vh = self._dims
        B, T, _ = hidden_states.shape
        zero = torch.zeros(B, hv, hk, vh, dtype=torch.float32, device=hidden_states.device)
        if Gdn2Mode(self.config.mode) == Gdn2Mode.Chunk:
            p, _ = self.project(hidden_states, None)
            normed = self._chunk_core(p, zero)
        elif hv == h or T == 1 or self.gva_mode == "grouped":
            normed, _ = self._recurrent_fused(hidden_states, None, zero)
        else:
            p, _ = self.project(hidden_states, None)
            normed = self._recurrent_projected(p, zero)
        return self._out_proj(normed)
