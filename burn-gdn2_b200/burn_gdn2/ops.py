"""Functional GDN-2 ops on CUDA tensors, each one C-ABI call into
libgdn2_b200.so.  Names, argument order and return values mirror the
reference crate (sehaxe/burn-gdn2 v0.5.1):

  chunk_wy_forward        src/forward.rs:44-278
  fused_recurrent_forward src/kernel/fused_recurrent.rs:11-56
  fused_recurrent_gdn2    src/kernel/fused_recurrent.rs:65-108
  short_conv_1d           src/short_conv.rs:22-65
  l2_normalize_4d         src/l2norm.rs:13-16
  rms_norm_gate_per_head  src/module.rs:501-517

Every op requires CUDA tensors and raises if it gets anything else: there is
no CPU or tensor-op fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import LIB, check

SHORT_CONV_KERNEL = 4  # src/short_conv.rs:5
SHORT_CONV_CACHE = 3  # src/short_conv.rs:7

_DT = {torch.float32: _lib.GDN2_DTYPE_F32, torch.bfloat16: _lib.GDN2_DTYPE_BF16}


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("burn_gdn2 ops run on the B200 CUDA kernels only; got a CPU tensor")


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DT:
        raise TypeError(f"unsupported dtype {dt}; use float32 or bfloat16")
    return _DT[dt]


def view4(t: Optional[torch.Tensor]) -> _lib.View:
    """gdn2_view of a 4-D tensor whose last dim is contiguous."""
    if t is None:
        return _lib.View()
    assert t.dim() == 4, t.shape
    if t.stride(3) != 1 and t.shape[3] > 1:
        raise ValueError("last dim must be contiguous")
    return _lib.View(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(device=None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _last_contig(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    t = t.to(dtype)
    if t.stride(-1) != 1 and t.shape[-1] > 1:
        t = t.contiguous()
    return t


def _expand_k(t: torch.Tensor, K: int) -> torch.Tensor:
    """g / b with a last dim of 1 broadcast over K (``k % g_dim``, src/forward.rs:149,173)."""
    if t.shape[-1] == K:
        return t
    if t.shape[-1] != 1:
        raise ValueError(f"last dim {t.shape[-1]} must be 1 or {K}")
    return t.expand(*t.shape[:-1], K).contiguous()


_PRECISION = {"f32": _lib.GDN2_PRECISION_F32, "bf16": _lib.GDN2_PRECISION_BF16}


def precision_code(precision: str) -> int:
    """'f32' (default): f32-grade intermediates; 'bf16': bf16 intermediates
    on the tensor cores for bf16 inputs (faster, ~3e-3 normwise error)."""
    if precision not in _PRECISION:
        raise ValueError(f"precision must be one of {sorted(_PRECISION)}, got {precision!r}")
    return _PRECISION[precision]


def chunk_args(q, k, v, g, b, w, state, out, scale, chunk_size, *, num_heads=None, grouped=False,
               gate=None, o_norm_weight=None, norm_eps=1e-5, precision="f32") -> _lib.ChunkArgs:
    """Fill gdn2_chunk_args.  q,k,g,b: [B,Hq,T,K]; v,w,out: [B,HV,T,V];
    gate: [B,HV,T,V] view or None; state: [B,HV,K,V] f32 contiguous."""
    B, Hq, T, K = q.shape
    HV, V = v.shape[1], v.shape[3]
    a = _lib.ChunkArgs()
    a.dims = _lib.Dims(B, T, num_heads if num_heads else Hq, HV, K, V)
    a.chunk_size = int(chunk_size)
    a.dtype = dtype_code(q.dtype)
    a.key_heads_grouped = int(grouped)
    a.fuse_epilogue = int(gate is not None)
    a.scale = float(scale)
    a.norm_eps = float(norm_eps)
    a.q, a.k, a.v, a.g, a.b, a.w = (view4(x) for x in (q, k, v, g, b, w))
    a.gate = view4(gate)
    a.o_norm_weight = None if o_norm_weight is None else o_norm_weight.data_ptr()
    a.state = state.data_ptr()
    a.out = view4(out)
    a.precision = precision_code(precision)
    return a


def chunk_workspace(a: _lib.ChunkArgs, device) -> torch.Tensor:
    nbytes = LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a))
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


def chunk_wy_forward(q, k, v, g, b, w, state, scale, chunk_size, precision="f32") -> Tuple[torch.Tensor, torch.Tensor]:
    """Chunked WY forward (src/forward.rs:44-278) on kernels (1) + (2).

    q,k,g,b: [B,HV,T,K] (g, b may have last dim 1); v,w: [B,HV,T,V];
    state [B,HV,K,V].  Returns (out [B,HV,T,V] in q's dtype, new state f32).
    precision: "f32" (f32-grade intermediates) or "bf16" (see precision_code).
    """
    _require_cuda(q, k, v, g, b, w, state)
    dt = q.dtype if q.dtype in _DT else torch.float32
    K = q.shape[3]
    q, k, v, w = (_last_contig(x, dt) for x in (q, k, v, w))
    b = _last_contig(_expand_k(b, K), dt)
    g = _last_contig(_expand_k(g, K), torch.float32)
    st = state.to(torch.float32).contiguous().clone()
    B, HV, T, _ = q.shape
    out = torch.empty(B, HV, T, v.shape[3], dtype=dt, device=q.device)
    a = chunk_args(q, k, v, g, b, w, st, out, scale, chunk_size, precision=precision)
    ws = chunk_workspace(a, q.device)
    check(LIB.gdn2_chunk_fwd(ctypes.byref(a), ptr(ws), ws.numel(), stream_handle(q.device)))
    return out, st


def recurrent_args(q, k, v, g, b, w, state, out, scale, *, num_heads=None, grouped=False, prologue=0,
                   conv_w=(None, None, None), conv_in=(None, None, None), conv_out=(None, None, None),
                   gate=None, o_norm_weight=None, norm_eps=1e-5, dtype=None) -> _lib.RecurrentArgs:
    B, Hq, T, K = q.shape
    HV, V = v.shape[1], v.shape[3]
    a = _lib.RecurrentArgs()
    a.dims = _lib.Dims(B, T, num_heads if num_heads else Hq, HV, K, V)
    a.dtype = dtype_code(dtype if dtype is not None else q.dtype)
    a.key_heads_grouped = int(grouped)
    a.prologue = int(prologue)
    a.fuse_epilogue = int(gate is not None)
    a.scale = float(scale)
    a.norm_eps = float(norm_eps)
    a.q, a.k, a.v, a.g, a.b, a.w = (view4(x) for x in (q, k, v, g, b, w))
    a.conv_w_q, a.conv_w_k, a.conv_w_v = (None if x is None else x.data_ptr() for x in conv_w)
    a.conv_q_in, a.conv_k_in, a.conv_v_in = (None if x is None else x.data_ptr() for x in conv_in)
    a.conv_q_out, a.conv_k_out, a.conv_v_out = (None if x is None else x.data_ptr() for x in conv_out)
    a.gate = view4(gate)
    a.o_norm_weight = None if o_norm_weight is None else o_norm_weight.data_ptr()
    a.state = state.data_ptr()
    a.out = view4(out)
    return a


def fused_recurrent_forward(q, k, v, g, b, w, state, scale) -> Tuple[torch.Tensor, torch.Tensor]:
    """Token-by-token scan (src/kernel/fused_recurrent.rs:11-56) on kernel (3):
    one launch, state on chip for all T tokens.  Returns (out [B,HV,T,V], state)."""
    _require_cuda(q, k, v, g, b, w, state)
    dt = q.dtype if q.dtype in _DT else torch.float32
    K = q.shape[3]
    q, k, v, w = (_last_contig(x, dt) for x in (q, k, v, w))
    b = _last_contig(_expand_k(b, K), dt)
    g = _last_contig(_expand_k(g, K), torch.float32)
    st = state.to(torch.float32).contiguous().clone()
    B, HV, T, _ = q.shape
    out = torch.empty(B, HV, T, v.shape[3], dtype=dt, device=q.device)
    a = recurrent_args(q, k, v, g, b, w, st, out, scale)
    check(LIB.gdn2_recurrent_fwd(ctypes.byref(a), stream_handle(q.device)))
    return out, st


def recurrent_backward(q, k, v, g, b, w, state, scale, d_out, d_state=None, *, num_heads=None):
    """Backward of the core recurrence (gdn2_recurrent_bwd, exact f32).

    q,k,g,b: [B,Hq,T,K] with Hq = HV, or Hq = num_heads key heads shared by
    groups of HV / Hq value heads; v,w,d_out: [B,HV,T,V]; state: [B,HV,K,V]
    initial state or None (zeros); d_state: dL/d(final state) or None.
    Returns (dq, dk, dv, dg, db, dw, d_state_in), f32, the key-side ones
    summed over each group back to [B,Hq,T,K].
    """
    _require_cuda(q, k, v, g, b, w, d_out)
    dt = q.dtype if q.dtype in _DT else torch.float32
    B, Hq, T, K = q.shape
    HV, V = v.shape[1], v.shape[3]
    grouped = Hq != HV
    if grouped and HV % Hq:
        raise ValueError(f"value heads {HV} not a multiple of key heads {Hq}")
    q, k, v, w, d_out = (_last_contig(x, dt) for x in (q, k, v, w, d_out))
    b = _last_contig(_expand_k(b, K), dt)
    g = _last_contig(_expand_k(g, K), torch.float32)
    st = None if state is None else state.to(torch.float32).contiguous()
    dst = None if d_state is None else d_state.to(torch.float32).contiguous()
    f32 = dict(dtype=torch.float32, device=q.device)
    dq, dk, dg, db = (torch.empty(B, HV, T, K, **f32) for _ in range(4))
    dv, dw = (torch.empty(B, HV, T, V, **f32) for _ in range(2))
    dh0 = torch.empty(B, HV, K, V, **f32)
    a = _lib.RecurrentBwdArgs()
    a.dims = _lib.Dims(B, T, Hq if grouped else HV, HV, K, V)
    a.dtype = dtype_code(dt)
    a.key_heads_grouped = int(grouped)
    a.scale = float(scale)
    a.q, a.k, a.v, a.g, a.b, a.w = (view4(x) for x in (q, k, v, g, b, w))
    a.state_in = None if st is None else st.data_ptr()
    a.d_out = view4(d_out)
    a.d_state_out = None if dst is None else dst.data_ptr()
    a.dq, a.dk, a.dv, a.dg, a.db, a.dw = (view4(x) for x in (dq, dk, dv, dg, db, dw))
    a.d_state_in = dh0.data_ptr()
    nbytes = LIB.gdn2_recurrent_bwd_workspace_bytes(ctypes.byref(a.dims))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    check(LIB.gdn2_recurrent_bwd(ctypes.byref(a), ptr(ws), ws.numel(), stream_handle(q.device)))
    if grouped:
        dq, dk, dg, db = (x.view(B, Hq, HV // Hq, T, K).sum(2) for x in (dq, dk, dg, db))
    return dq, dk, dv, dg, db, dw, dh0


def chunk_trajectory(q, k, v, g, b, w, state, chunk_size, with_v_new=True):
    """Trajectory export (gdn2_chunk_trajectory; the crate's
    gdn2_chunk_trajectory_export_kernel, src/kernel/chunk_cube.rs:613-734):
    the state entering every chunk [B,HV,ceil(T/C),K,V] f32 and v_new per
    token [B,HV,T,V] f32 (None unless with_v_new), exact f32.  Shapes as
    fused_recurrent_forward; state None = zeros (not modified)."""
    _require_cuda(q, k, v, g, b, w)
    dt = q.dtype if q.dtype in _DT else torch.float32
    K = q.shape[3]
    q, k, v, w = (_last_contig(x, dt) for x in (q, k, v, w))
    b = _last_contig(_expand_k(b, K), dt)
    g = _last_contig(_expand_k(g, K), torch.float32)
    B, HV, T, _ = q.shape
    V = v.shape[3]
    st = None if state is None else state.to(torch.float32).contiguous()
    states = torch.empty(B, HV, (T + chunk_size - 1) // chunk_size, K, V, dtype=torch.float32, device=q.device)
    vnew = torch.empty(B, HV, T, V, dtype=torch.float32, device=q.device) if with_v_new else None
    a = recurrent_args(q, k, v, g, b, w, st if st is not None else states, vnew, 1.0)
    a.state = None if st is None else st.data_ptr()
    a.out = _lib.View()
    check(LIB.gdn2_chunk_trajectory(ctypes.byref(a), int(chunk_size), ptr(states), view4(vnew),
                                    stream_handle(q.device)))
    return states, vnew


class GatedDeltaCore(torch.autograd.Function):
    """Differentiable core: forward on the chunked kernels (1) + (2), f32-grade
    (or the recurrent kernel (3) for T <= 64), backward on gdn2_recurrent_bwd.

    apply(q, k, v, g, b, w, state, scale, chunk_size) -> (out [B,HV,T,V], new state f32).
    q,k,g,b: [B,HV,T,K] (g, b last dim K); gradients flow to q, k, v, g, b, w
    and the initial state; the new state's gradient is taken into account.
    """

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, state, scale, chunk_size):
        s0 = state if state is not None else torch.zeros(q.shape[0], v.shape[1], q.shape[3], v.shape[3],
                                                          dtype=torch.float32, device=q.device)
        if q.shape[2] <= 64:
            out, st = fused_recurrent_forward(q, k, v, g, b, w, s0, scale)
        else:
            out, st = chunk_wy_forward(q, k, v, g, b, w, s0, scale, chunk_size)
        ctx.save_for_backward(q, k, v, g, b, w, state)
        ctx.scale = scale
        return out, st

    @staticmethod
    def backward(ctx, d_out, d_state):
        q, k, v, g, b, w, state = ctx.saved_tensors
        if d_out is None:
            d_out = torch.zeros(v.shape, dtype=v.dtype, device=v.device)
        dq, dk, dv, dg, db, dw, dh0 = recurrent_backward(q, k, v, g, b, w, state, ctx.scale, d_out, d_state)
        cast = lambda gr, x: gr.to(x.dtype)
        return (cast(dq, q), cast(dk, k), cast(dv, v), cast(dg, g), cast(db, b), cast(dw, w),
                None if state is None else cast(dh0, state), None, None)


def fused_recurrent_gdn2(q, k, v, g, b, w, state: Optional[torch.Tensor], scale, update_state: bool):
    """Dispatcher of src/kernel/fused_recurrent.rs:65-108.

    update_state: run the scan (any T; T == 1 is the decode step) and return
    (out [B,HV,T,V], new state).  Otherwise the read-only branch
    (:101-104): out = scale * q S, permuted to [B,T,HV,V], state unchanged.
    """
    B, HV, T, K = q.shape
    V = v.shape[3]
    s = state if state is not None else torch.zeros(B, HV, K, V, device=q.device, dtype=torch.float32)
    if update_state:
        return fused_recurrent_forward(q, k, v, g, b, w, s, scale)
    out = (q.float() @ s * scale).permute(0, 2, 1, 3)
    return out, s


def short_conv_1d(x, weight, cache=None):
    """Causal depthwise conv (kernel 4) + SiLU (src/short_conv.rs:22-65).
    x [B,T,C]; weight [C,4]; cache [B,3,C] or None.  Returns (y, new_cache f32)."""
    _require_cuda(x, weight, cache)
    dt = x.dtype if x.dtype in _DT else torch.float32
    x = x.to(dt).contiguous()
    Bn, T, C = x.shape
    y = torch.empty_like(x)
    w32 = weight.to(torch.float32).contiguous()
    cin = None if cache is None else cache.to(torch.float32).contiguous()
    cout = torch.empty(Bn, SHORT_CONV_CACHE, C, dtype=torch.float32, device=x.device)
    check(LIB.gdn2_short_conv(Bn, T, C, dtype_code(dt), ptr(x), ptr(w32), ptr(cin), ptr(cout), ptr(y),
                              stream_handle(x.device)))
    return y, cout


def project_activations(q_raw, k_raw, v_raw, b_raw, w_raw, f_raw, *, batch, num_heads, head_k_dim, num_v_heads,
                        head_v_dim, a_log, dt_bias, conv_w=None, conv_in=None, allow_neg_eigval=False,
                        min_decay=None, decay_factors=None):
    """Elementwise part of ``project`` (src/module.rs:381-498) in one launch:
    q, k = L2(SiLU(conv4(raw))), v = SiLU(conv4(v_raw)), b, w = sigmoid
    (b x 2 with neg-eig), g = -exp(A_log) softplus(f_raw + dt_bias) (f32,
    min_decay remap).  Raw inputs: [B*T, C] row-major views (unit column
    stride, any row stride, e.g. column slices of one GEMM output).
    ``conv_w`` = (q, k, v) [C,4] weights or None (no short conv);
    ``conv_in`` = (q, k, v) [B,3,C] caches or None (replicate token 0).
    Returns (q, k, v, b, w, g) as [B*T, C] tensors and the new conv caches
    (or None)."""
    raws = (q_raw, k_raw, v_raw, b_raw, w_raw, f_raw)
    _require_cuda(*raws)
    dt = q_raw.dtype
    for r in raws:
        if r.dtype != dt or r.dim() != 2 or r.stride(1) != 1:
            raise ValueError("project_activations: raw inputs must be 2-D, unit column stride, one dtype")
    N = q_raw.shape[0]
    kd, vd = num_heads * head_k_dim, num_v_heads * head_v_dim
    dev = q_raw.device
    a = _lib.PrologueArgs()
    a.dims = _lib.Dims(batch, N // batch, num_heads, num_v_heads, head_k_dim, head_v_dim)
    a.dtype = dtype_code(dt)
    a.use_short_conv = int(conv_w is not None)
    a.allow_neg_eigval = int(bool(allow_neg_eigval))
    a.min_decay = -1.0 if min_decay is None else float(min_decay)
    for name, r in zip(("q", "k", "v", "b", "w", "f"), raws):
        setattr(a, name + "_raw", r.data_ptr())
        setattr(a, "ld_" + name, r.stride(0))
    f32 = lambda t: None if t is None else t.to(dev, torch.float32).contiguous()
    keep = []
    conv_out = None
    if conv_w is not None:
        cw = [f32(w) for w in conv_w]
        keep += cw
        a.conv_w_q, a.conv_w_k, a.conv_w_v = (t.data_ptr() for t in cw)
        if conv_in is not None:
            ci = [f32(c) for c in conv_in]
            keep += ci
            a.conv_q_in, a.conv_k_in, a.conv_v_in = (t.data_ptr() for t in ci)
        conv_out = tuple(torch.empty(batch, SHORT_CONV_CACHE, n, dtype=torch.float32, device=dev)
                         for n in (kd, kd, vd))
        a.conv_q_out, a.conv_k_out, a.conv_v_out = (t.data_ptr() for t in conv_out)
    al, dtb = f32(a_log), f32(dt_bias)
    keep += [al, dtb]
    a.a_log, a.dt_bias = al.data_ptr(), dtb.data_ptr()
    if min_decay is not None:
        dfac = f32(decay_factors).reshape(-1)
        keep.append(dfac)
        a.decay_factors = dfac.data_ptr()
    q = torch.empty(N, kd, dtype=dt, device=dev)
    k = torch.empty_like(q)
    b = torch.empty_like(q)
    v = torch.empty(N, vd, dtype=dt, device=dev)
    w = torch.empty_like(v)
    g = torch.empty(N, kd, dtype=torch.float32, device=dev)
    a.q, a.k, a.v, a.b, a.w, a.g = (t.data_ptr() for t in (q, k, v, b, w, g))
    check(LIB.gdn2_project_activations(ctypes.byref(a), stream_handle(dev)))
    return (q, k, v, b, w, g), conv_out


def l2_normalize_4d(x, eps=1e-6):
    """x / sqrt(sum_K x^2 + eps) (src/l2norm.rs:13-16)."""
    xf = x.float()
    return (xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


def rms_norm_gate_per_head(x, gate, weight, eps):
    """x / sqrt(mean_V x^2 + eps) * weight * silu(gate) (src/module.rs:501-517).
    x, gate: [B,T,HV,V] (any strides with V contiguous); weight [V]."""
    _require_cuda(x, gate, weight)
    dt = x.dtype if x.dtype in _DT else torch.float32
    x = _last_contig(x, dt)
    gate = _last_contig(gate, dt)
    B, T, HV, V = x.shape
    out = torch.empty(B, T, HV, V, dtype=dt, device=x.device)
    dims = _lib.Dims(B, T, HV, HV, 1, V)
    w32 = weight.to(torch.float32).contiguous()
    perm = lambda t: t.permute(0, 2, 1, 3)  # [B,HV,T,V] views
    check(LIB.gdn2_rms_norm_gate(ctypes.byref(dims), dtype_code(dt), view4(perm(x)), view4(perm(gate)), ptr(w32),
                                 float(eps), view4(perm(out)), stream_handle(x.device)))
    return out
