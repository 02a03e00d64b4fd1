"""GPU parity of the core kernels against the CPU oracle (float64), through
the C ABI (burn_gdn2.ops -> libgdn2_b200.so).

Tolerances (north star): f32 inputs rel 1e-3 / abs 1e-4 elementwise; bf16
inputs with f32 accumulation rel 2e-2 elementwise with an absolute floor of
1e-2 x RMS of the reference (helpers.assert_close_bf16).  bf16 cases feed the
oracle the same bf16-rounded inputs.  The opt-in bf16-intermediate chunk
path (precision="bf16") is held to its own documented accuracy
(helpers.assert_close_bf16_intermediates).
"""
import ctypes

import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import F32_TOL, assert_close, assert_close_bf16, assert_close_bf16_intermediates

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _to_dev(arrs, dtype):
    return {k: torch.tensor(v, dtype=torch.float32 if k == "g" else dtype, device=DEV) for k, v in arrs.items()}


def _oracle_inputs(dev_arrs):
    return {k: v.detach().float().cpu().numpy().astype(np.float64) for k, v in dev_arrs.items()}


def _check(got, want, dtype, what):
    if dtype == torch.float32:
        assert_close(got, want, what=what, **F32_TOL)
    else:
        assert_close_bf16(got, want, what=what)


CORE_SHAPES = [
    # B, HV, T, K, V
    (2, 3, 96, 8, 8),
    (2, 3, 130, 16, 8),
    (1, 4, 70, 16, 24),
    (1, 2, 200, 64, 64),
    (1, 2, 129, 128, 128),
    (1, 2, 100, 128, 256),
]


@pytest.mark.parametrize("shape", CORE_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_recurrent_matches_oracle(shape, dtype):
    import burn_gdn2 as bg

    B, HV, T, K, V = shape
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=11, dtype=np.float32)
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, dtype)
    s0 = np.random.default_rng(12).standard_normal((B, HV, K, V)).astype(np.float32)
    o, s = bg.fused_recurrent_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"],
                                      torch.tensor(s0, device=DEV), K ** -0.5)
    ref = _oracle_inputs(d)
    o_ref, s_ref = O.fused_recurrent_forward(ref["q"], ref["k"], ref["v"], ref["g"], ref["b"], ref["w"],
                                             s0.astype(np.float64), K ** -0.5)
    _check(o.float().cpu().numpy(), o_ref, dtype, "out")
    _check(s.cpu().numpy(), s_ref, torch.float32 if dtype == torch.float32 else dtype, "state")


@pytest.mark.parametrize("shape", CORE_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("chunk", [64, 16])
def test_chunk_matches_oracle(shape, dtype, chunk):
    import burn_gdn2 as bg

    B, HV, T, K, V = shape
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=21, dtype=np.float32)
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, dtype)
    s0 = np.random.default_rng(22).standard_normal((B, HV, K, V)).astype(np.float32)
    o, s = bg.chunk_wy_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"],
                               torch.tensor(s0, device=DEV), K ** -0.5, chunk)
    ref = _oracle_inputs(d)
    o_ref, s_ref = O.chunk_wy_forward(ref["q"], ref["k"], ref["v"], ref["g"], ref["b"], ref["w"],
                                      s0.astype(np.float64), K ** -0.5, chunk)
    _check(o.float().cpu().numpy(), o_ref, dtype, "out")
    _check(s.cpu().numpy(), s_ref, dtype, "state")


@pytest.mark.parametrize("decay", [(-0.3, -0.02), (-5.0, -0.5)])
@pytest.mark.parametrize("chunk", [16, 64, 4, 30])
def test_stable_chunk_gpu(decay, chunk):
    """tests/stable_chunk.rs:11-72 on the GPU: scalar-broadcast g and b
    ([B,H,T,1]), chunk sizes 16 and 64 (plus 4 and 30), scale 1, 1e-3."""
    import burn_gdn2 as bg

    rng = np.random.default_rng(31)
    B, H, T, K, V = 2, 3, 96, 8, 8
    q = rng.standard_normal((B, H, T, K))
    kr = rng.standard_normal((B, H, T, K))
    k = kr / np.sqrt((kr * kr).sum(-1, keepdims=True))
    v = rng.standard_normal((B, H, T, V))
    g = rng.uniform(decay[0], decay[1], (B, H, T, 1))
    b = rng.uniform(0.0, 1.0, (B, H, T, 1))
    w = rng.standard_normal((B, H, T, V))
    t = lambda x: torch.tensor(x, dtype=torch.float32, device=DEV)
    s0 = np.zeros((B, H, K, V))
    o_ref, s_ref = O.fused_recurrent_forward(q, k, v, g, b, w, s0, 1.0)
    o, s = bg.chunk_wy_forward(t(q), t(k), t(v), t(g), t(b), t(w), t(s0), 1.0, chunk)
    assert np.abs(o.cpu().numpy() - o_ref).max() < 1e-3
    assert np.abs(s.cpu().numpy() - s_ref).max() < 1e-3
    o2, s2 = bg.fused_recurrent_forward(t(q), t(k), t(v), t(g), t(b), t(w), t(s0), 1.0)
    assert np.abs(o2.cpu().numpy() - o_ref).max() < 1e-3


def test_chunk_real_decay_t130_gpu():
    """tests/test_chunk.rs:200-256: T=130 (partial chunk), per-channel decay
    U(-0.15,-0.01), K=16, V=8, random S0, scale 0.125; 1e-4."""
    import burn_gdn2 as bg

    rng = np.random.default_rng(41)
    B, H, T, K, V = 2, 3, 130, 16, 8
    g = rng.uniform(-0.15, -0.01, (B, H, T, K))
    q = rng.standard_normal((B, H, T, K))
    kr = rng.standard_normal((B, H, T, K))
    k = kr / np.sqrt((kr ** 2).sum(-1, keepdims=True))
    v = rng.standard_normal((B, H, T, V))
    e = rng.uniform(0.0, 1.0, (B, H, T, K))
    w = rng.standard_normal((B, H, T, V))
    s0 = rng.standard_normal((B, H, K, V))
    t = lambda x: torch.tensor(x, dtype=torch.float32, device=DEV)
    o_ref, s_ref = O.fused_recurrent_forward(q, k, v, g, e, w, s0, 0.125)
    o, s = bg.chunk_wy_forward(t(q), t(k), t(v), t(g), t(e), t(w), t(s0), 0.125, 64)
    assert np.abs(o.cpu().numpy() - o_ref).max() < 1e-4
    assert np.abs(s.cpu().numpy() - s_ref).max() < 1e-4


def test_decode_steps_equal_chunked_forward():
    """North star: token-by-token decode reproduces one chunked forward
    (f32, rel 1e-3 / abs 1e-4), here at K = V = 128 over 3 chunks."""
    import burn_gdn2 as bg

    B, HV, T, K, V = 2, 4, 150, 128, 128
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=51, dtype=np.float32)
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, torch.float32)
    s0 = torch.zeros(B, HV, K, V, device=DEV)
    oc, sc = bg.chunk_wy_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], s0, K ** -0.5, 64)
    st = s0.clone()
    outs = []
    for t in range(T):
        sl = {k: v[:, :, t:t + 1] for k, v in d.items()}
        o, st = bg.fused_recurrent_forward(sl["q"], sl["k"], sl["v"], sl["g"], sl["b"], sl["w"], st, K ** -0.5)
        outs.append(o)
    od = torch.cat(outs, 2)
    assert_close(od.cpu().numpy(), oc.cpu().numpy(), what="out", **F32_TOL)
    assert_close(st.cpu().numpy(), sc.cpu().numpy(), what="state", **F32_TOL)


def test_chunk_intra_inter_split_equals_fused_call():
    """gdn2_chunk_intra + gdn2_chunk_inter == gdn2_chunk_fwd, bit for bit."""
    import ctypes
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    B, HV, T, K, V = 1, 2, 200, 64, 64
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=61, dtype=np.float32)
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, torch.float32)
    res = []
    for split in (False, True):
        st = torch.zeros(B, HV, K, V, device=DEV)
        out = torch.empty(B, HV, T, V, device=DEV)
        a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], st, out, K ** -0.5, 64)
        ws = ops.chunk_workspace(a, DEV)
        s = ops.stream_handle()
        if split:
            bg._lib.check(bg.LIB.gdn2_chunk_intra(ctypes.byref(a), ops.ptr(ws), ws.numel(), s))
            bg._lib.check(bg.LIB.gdn2_chunk_inter(ctypes.byref(a), ops.ptr(ws), ws.numel(), s))
        else:
            bg._lib.check(bg.LIB.gdn2_chunk_fwd(ctypes.byref(a), ops.ptr(ws), ws.numel(), s))
        torch.cuda.synchronize()
        res.append((out.cpu(), st.cpu()))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


def _chunk_full(d, gate, onw, s0, H, grouped, precision="f32"):
    """gdn2_chunk_fwd with the fused gated RMS-norm epilogue.  d: q,k,g,b
    [B,Hq,T,K] and v,w [B,HV,T,V] device views; gate [B,T,HV,V] storage.
    Returns (out [B,T,HV,V], state)."""
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    B, _, T, K = d["q"].shape
    HV, V = d["v"].shape[1], d["v"].shape[3]
    st = s0.clone()
    out = torch.empty(B, T, HV, V, device=DEV, dtype=d["v"].dtype)
    a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], st, out.permute(0, 2, 1, 3), K ** -0.5, 64,
                       num_heads=H, grouped=grouped, gate=gate.permute(0, 2, 1, 3), o_norm_weight=onw,
                       norm_eps=1e-5, precision=precision)
    ws = ops.chunk_workspace(a, DEV)
    bg._lib.check(bg.LIB.gdn2_chunk_fwd(ctypes.byref(a), ops.ptr(ws), ws.numel(), ops.stream_handle()))
    torch.cuda.synchronize()
    return out, st


def _oracle_full(d, gate, onw, s0, rep=1):
    """f64 oracle of _chunk_full on the same (dtype-rounded) inputs: key-side
    heads repeated per value head (np.repeat, the grouped mapping)."""
    r = lambda x: x.float().cpu().numpy().astype(np.float64)
    kv = lambda x: np.repeat(r(x), rep, axis=1)
    K = d["q"].shape[3]
    o_ref, s_ref = O.chunk_wy_forward(kv(d["q"]), kv(d["k"]), r(d["v"]), kv(d["g"]), kv(d["b"]), r(d["w"]),
                                      r(s0), K ** -0.5, 64)
    y_ref = O.rms_norm_gate_per_head(o_ref.transpose(0, 2, 1, 3), r(gate), r(onw), 1e-5)
    return y_ref, s_ref


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_chunk_config2_head_shape_vs_oracle(dtype):
    """BASELINE config-2 head shape (K = V = 128, T = 4096, chunk 64, the
    module's value laws) on two value heads with the fused gated RMS norm and
    a random initial state, vs the f64 oracle: the gated output elementwise
    and the final state."""
    B, HV, T, K, V = 1, 2, 4096, 128, 128
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=71, dtype=np.float32, decay=(-1.6, -0.001))
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, dtype)
    gate = torch.tensor(arrs["gate"], device=DEV, dtype=dtype)
    onw = torch.tensor(np.random.default_rng(72).uniform(0.5, 1.5, V).astype(np.float32), device=DEV)
    s0 = torch.tensor(np.random.default_rng(73).standard_normal((B, HV, K, V)).astype(np.float32), device=DEV)
    y, st = _chunk_full(d, gate, onw, s0, HV, False)
    y_ref, s_ref = _oracle_full(d, gate, onw, s0)
    _check(y.float().cpu().numpy(), y_ref, dtype, "gated out")
    _check(st.cpu().numpy(), s_ref, torch.float32 if dtype == torch.float32 else dtype, "state")
    import burn_gdn2 as bg
    assert bg._lib.read_device_errors() == 0


def test_short_conv_and_rms_norm_gate_kernels():
    import burn_gdn2 as bg

    rng = np.random.default_rng(81)
    x = rng.standard_normal((2, 9, 40)).astype(np.float32)
    wc = rng.uniform(-0.5, 0.5, (40, 4)).astype(np.float32)
    cache = rng.standard_normal((2, 3, 40)).astype(np.float32)
    t = lambda a: torch.tensor(a, device=DEV)
    for c in (None, cache):
        y, nc = bg.short_conv_1d(t(x), t(wc), None if c is None else t(c))
        yr, ncr = O.short_conv_1d(x.astype(np.float64), wc.astype(np.float64),
                                  None if c is None else c.astype(np.float64))
        assert_close(y.cpu().numpy(), yr, what="conv", **F32_TOL)
        assert_close(nc.cpu().numpy(), ncr, what="cache", **F32_TOL)
    o = rng.standard_normal((2, 5, 3, 24)).astype(np.float32)
    gate = rng.standard_normal((2, 5, 3, 24)).astype(np.float32)
    wn = rng.uniform(0.5, 1.5, 24).astype(np.float32)
    y = bg.rms_norm_gate_per_head(t(o), t(gate), t(wn), 1e-5)
    yr = O.rms_norm_gate_per_head(o.astype(np.float64), gate.astype(np.float64), wn.astype(np.float64), 1e-5)
    assert_close(y.cpu().numpy(), yr, what="rms", **F32_TOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_chunk_split_path_one_and_two_ctas_per_chain(dtype):
    """K = V = 128 on the split-operand path with the fused gated RMS norm,
    once with more chains than half the SMs (one CTA per chain: B = 2,
    HV = 40) and once with few chains (each chain's value columns over two
    64-column CTAs that exchange the norm's row sums: B = 1, HV = 3); both
    vs the f64 oracle, the gated output elementwise and the final state."""
    import burn_gdn2 as bg

    for B, HV, T in ((2, 40, 130), (1, 3, 200)):
        K = V = 128
        arrs = O.make_core_inputs(B, HV, T, K, V, seed=77, dtype=np.float32, decay=(-1.6, -0.001))
        d = _to_dev({k: arrs[k] for k in "qkvgbw"}, dtype)
        gate = torch.tensor(arrs["gate"], device=DEV, dtype=dtype)
        onw = torch.tensor(np.random.default_rng(78).uniform(0.5, 1.5, V).astype(np.float32), device=DEV)
        s0 = torch.tensor(np.random.default_rng(79).standard_normal((B, HV, K, V)).astype(np.float32), device=DEV)
        y, st = _chunk_full(d, gate, onw, s0, HV, False)
        y_ref, s_ref = _oracle_full(d, gate, onw, s0)
        _check(y.float().cpu().numpy(), y_ref, dtype, "gated out")
        _check(st.cpu().numpy(), s_ref, torch.float32 if dtype == torch.float32 else dtype, "state")
    assert bg._lib.read_device_errors() == 0


@pytest.mark.parametrize("reserve", [0, 64])
@pytest.mark.parametrize("shape", [(1, 3, 1600, 128, 128), (1, 1, 2048, 128, 256), (2, 12, 2048, 128, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_chunk_state_scan_segments(shape, dtype, reserve):
    """Few long chains: the split-operand inter kernel cuts each chain into
    segments (3 of 9, 9 and 7 chunks for 3 chains at V = 128; 4 of 8 at
    V = 256; 3 for 24 chains), computes every segment's end state from zero
    and its state transition in parallel, chains the start states, then runs
    the segments in parallel.  With the fused gated RMS norm and a random
    initial state, vs the f64 oracle: gated output elementwise, final state;
    also with 64 SMs reserved (gdn2_set_reserved_sms: a smaller intra grid,
    and for the 24 chains no scan but 64-column cluster pairs)."""
    import burn_gdn2 as bg

    prev = bg.LIB.gdn2_set_reserved_sms(reserve)
    try:
        _scan_case(shape, dtype)
    finally:
        bg.LIB.gdn2_set_reserved_sms(prev)


def _scan_case(shape, dtype):
    import burn_gdn2 as bg

    B, HV, T, K, V = shape
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=87, dtype=np.float32, decay=(-0.4, -0.001))
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, dtype)
    gate = torch.tensor(arrs["gate"], device=DEV, dtype=dtype)
    onw = torch.tensor(np.random.default_rng(88).uniform(0.5, 1.5, V).astype(np.float32), device=DEV)
    s0 = torch.tensor(np.random.default_rng(89).standard_normal((B, HV, K, V)).astype(np.float32), device=DEV)
    y, st = _chunk_full(d, gate, onw, s0, HV, False)
    y_ref, s_ref = _oracle_full(d, gate, onw, s0)
    _check(y.float().cpu().numpy(), y_ref, dtype, "gated out")
    _check(st.cpu().numpy(), s_ref, torch.float32 if dtype == torch.float32 else dtype, "state")
    assert bg._lib.read_device_errors() == 0


@pytest.mark.parametrize("shape", [(2, 3, 190, 128, 64), (1, 2, 64, 128, 128), (2, 2, 1, 128, 128),
                                   (1, 2, 200, 128, 256)])
@pytest.mark.parametrize("precision", ["f32", "bf16"])
def test_chunk_tensor_core_path_bf16(shape, precision):
    """bf16, K = 128, chunk 64 (the tcgen05 paths: split-operand for
    precision "f32", bf16 intermediates for "bf16"), V = 64 / 128 / 256, full and
    partial chunks including T = 1; permuted [B,T,H,D] storage views like
    the module's; random initial state; vs the f64 oracle."""
    import burn_gdn2 as bg

    B, HV, T, K, V = shape
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=91, dtype=np.float32)
    # storage [B,T,H,D], passed as [B,H,T,D] views
    d = {n: torch.tensor(np.ascontiguousarray(a.transpose(0, 2, 1, 3)), device=DEV,
                         dtype=torch.float32 if n == "g" else torch.bfloat16).permute(0, 2, 1, 3)
         for n, a in arrs.items() if n in "qkvgbw"}
    s0 = np.random.default_rng(92).standard_normal((B, HV, K, V)).astype(np.float32) * 0.5
    o, s = bg.chunk_wy_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"],
                               torch.tensor(s0, device=DEV), K ** -0.5, 64, precision=precision)
    ref = {n: v.float().cpu().numpy().astype(np.float64) for n, v in d.items()}
    o_ref, s_ref = O.chunk_wy_forward(ref["q"], ref["k"], ref["v"], ref["g"], ref["b"], ref["w"],
                                      s0.astype(np.float64), K ** -0.5, 64)
    chk = assert_close_bf16 if precision == "f32" else assert_close_bf16_intermediates
    chk(o.float().cpu().numpy(), o_ref, what="out")
    chk(s.cpu().numpy(), s_ref, what="state")


@pytest.mark.parametrize("V,precision", [(128, "f32"), (128, "bf16"), (256, "f32"), (256, "bf16")])
def test_chunk_tensor_core_path_is_deterministic(V, precision):
    """The tensor-core chunk paths have no atomics and no order-dependent
    reductions: two calls on the same inputs give bit-identical outputs and
    states (V = 256 runs each chain as two 128-column CTAs)."""
    import burn_gdn2 as bg

    B, HV, T, K = 2, 3, 300, 128
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=95, dtype=np.float32)
    d = {n: torch.tensor(a, device=DEV, dtype=torch.float32 if n == "g" else torch.bfloat16)
         for n, a in arrs.items() if n in "qkvgbw"}
    s0 = torch.tensor(np.random.default_rng(96).standard_normal((B, HV, K, V)).astype(np.float32) * 0.5, device=DEV)
    runs = [bg.chunk_wy_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], s0.clone(), K ** -0.5, 64,
                                precision=precision) for _ in range(2)]
    assert torch.equal(runs[0][0], runs[1][0])
    assert torch.equal(runs[0][1], runs[1][1])
    assert torch.isfinite(runs[0][0].float()).all()


@pytest.mark.parametrize("precision", ["f32", "bf16"])
def test_chunk_tensor_core_grouped_heads_and_epilogue(precision):
    """GVA without a materialised repeat (key_heads_grouped = 1: value head
    hv reads key head hv // 2) and the fused gated RMS-norm epilogue, on the
    tcgen05 paths, vs the oracle (np.repeat over heads + rms_norm_gate).
    The default path's gated output is checked elementwise; the
    bf16-intermediate path's normwise and against its largest magnitude (the
    RMS norm rescales a row whose pre-norm output is a cancellation to O(1),
    keeping its bf16 relative error at full scale)."""
    import burn_gdn2 as bg

    B, H, HV, T, K, V = 2, 2, 4, 130, 128, 128
    rng = np.random.default_rng(93)
    kq = O.make_core_inputs(B, H, T, K, V, seed=94, dtype=np.float32)
    kv = O.make_core_inputs(B, HV, T, K, V, seed=95, dtype=np.float32)
    t = lambda a, dt=torch.bfloat16: torch.tensor(a, device=DEV, dtype=dt)
    d = dict(q=t(kq["q"]), k=t(kq["k"]), b=t(kq["b"]), g=t(kq["g"], torch.float32), v=t(kv["v"]), w=t(kv["w"]))
    gate = t(rng.standard_normal((B, T, HV, V)).astype(np.float32))
    onw = t(rng.uniform(0.5, 1.5, V).astype(np.float32), torch.float32)
    y, st = _chunk_full(d, gate, onw, torch.zeros(B, HV, K, V, device=DEV), H, True, precision)
    y_ref, s_ref = _oracle_full(d, gate, onw, torch.zeros(B, HV, K, V), rep=HV // H)
    y = y.float().cpu().numpy()
    if precision == "f32":
        assert_close_bf16(y, y_ref, what="gated out")
        assert_close_bf16(st.cpu().numpy(), s_ref, what="state")
    else:
        assert np.linalg.norm(y - y_ref) / np.linalg.norm(y_ref) <= 1e-2
        assert np.abs(y - y_ref).max() <= 0.05 * np.abs(y_ref).max()
        assert_close_bf16_intermediates(st.cpu().numpy(), s_ref, what="state")
    assert bg._lib.read_device_errors() == 0


def test_chunk_config4_features_bf16():
    """BASELINE config-4 core features at small size: 2 key heads grouped
    over 4 value heads (value head hv reads key head hv // 2), K = 128,
    V = 256 (with the default precision: the split-operand tensor-core
    kernels, each chain as a 2-CTA cluster of 128-column halves that exchange
    the gated RMS norm's row sums), neg-eig b in [0, 2], g after the
    min_decay 0.9 remap, a partial last chunk; bf16 vs the f64 oracle."""
    import ctypes
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    B, H, HV, T, K, V = 2, 2, 4, 150, 128, 256
    rng = np.random.default_rng(96)
    kq = O.make_core_inputs(B, H, T, K, V, seed=97, dtype=np.float32)
    kv = O.make_core_inputs(B, HV, T, K, V, seed=98, dtype=np.float32)
    gate = rng.standard_normal((B, T, HV, V)).astype(np.float32)
    onw = rng.uniform(0.5, 1.5, V).astype(np.float32)
    fac = (1.0 / (1.0 + np.exp(-2.0))) * (1.0 - 0.9)
    g_remap = np.log(fac * np.exp(kq["g"].astype(np.float64)) + 0.9).astype(np.float32)
    t = lambda a, dt=torch.bfloat16: torch.tensor(a, device=DEV, dtype=dt)
    q, k, b = t(kq["q"]), t(kq["k"]), t(2.0 * kq["b"])
    g = t(g_remap, torch.float32)
    v, w = t(kv["v"]), t(kv["w"])
    gt = t(gate)
    st = torch.zeros(B, HV, K, V, device=DEV)
    out = torch.empty(B, T, HV, V, device=DEV, dtype=torch.bfloat16)
    a = ops.chunk_args(q, k, v, g, b, w, st, out.permute(0, 2, 1, 3), K ** -0.5, 64, num_heads=H, grouped=True,
                       gate=gt.permute(0, 2, 1, 3), o_norm_weight=t(onw, torch.float32), norm_eps=1e-5)
    ws = ops.chunk_workspace(a, DEV)
    bg._lib.check(bg.LIB.gdn2_chunk_fwd(ctypes.byref(a), ops.ptr(ws), ws.numel(), ops.stream_handle()))
    torch.cuda.synchronize()
    r = lambda x: x.float().cpu().numpy().astype(np.float64)
    rep = lambda x: np.repeat(x, HV // H, axis=1)
    o_ref, s_ref = O.chunk_wy_forward(rep(r(q)), rep(r(k)), r(v), rep(r(g)), rep(r(b)), r(w),
                                      np.zeros((B, HV, K, V)), K ** -0.5, 64)
    y_ref = O.rms_norm_gate_per_head(o_ref.transpose(0, 2, 1, 3), r(gt), onw.astype(np.float64), 1e-5)
    y = out.float().cpu().numpy()
    assert_close_bf16(y, y_ref, what="gated out")
    assert_close_bf16(st.cpu().numpy(), s_ref, what="state")
    assert bg._lib.read_device_errors() == 0


def test_chunk_long_sequence_config5_bf16():
    """BASELINE config-5 sequence length (T = 65536, 1024 chunks per chain)
    on the split-operand tensor-core path, one value head with the fused
    gated RMS norm and a random initial state, vs the f64 oracle: the gated
    output elementwise and the final state."""
    B, HV, T, K, V = 1, 1, 65536, 128, 128
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=99, dtype=np.float32, decay=(-1.6, -0.001))
    d = _to_dev({k: arrs[k] for k in "qkvgbw"}, torch.bfloat16)
    gate = torch.tensor(arrs["gate"], device=DEV, dtype=torch.bfloat16)
    onw = torch.ones(V, device=DEV)
    s0 = torch.tensor(np.random.default_rng(100).standard_normal((B, HV, K, V)).astype(np.float32) * 0.5,
                      device=DEV)
    y, st = _chunk_full(d, gate, onw, s0, HV, False)
    y_ref, s_ref = _oracle_full(d, gate, onw, s0)
    assert_close_bf16(y.float().cpu().numpy(), y_ref, what="gated out")
    assert_close_bf16(st.cpu().numpy(), s_ref, what="state")
    import burn_gdn2 as bg
    assert bg._lib.read_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_benched_configuration_vs_oracle(dtype):
    """The decode step as BASELINE config 3 runs it (kernel (3), K = V = 128,
    grouped key heads, prologue = 1: raw projections through the kernel-4
    short conv with the [B,3,C] caches updated in place, SiLU and L2 norm;
    the fused gated RMS-norm epilogue; the state updated in place), three
    steps in a row, vs the oracle's short_conv_1d / l2_normalize_4d /
    fused_recurrent_forward / rms_norm_gate_per_head (the calls of
    src/module.rs:224-316 with src/kernel/fused_recurrent.rs:11-56)."""
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    B, H, K, V = 4, 4, 128, 128
    HV, kd, vd = H, H * K, H * V
    rng = np.random.default_rng(111)
    f = lambda *sh: rng.standard_normal(sh).astype(np.float32)
    S = f(B, HV, K, V) * 0.5
    caches = [f(B, 3, kd), f(B, 3, kd), f(B, 3, vd)]
    cw = [rng.uniform(-0.5, 0.5, (n, 4)).astype(np.float32) for n in (kd, kd, vd)]
    onw = rng.uniform(0.5, 1.5, V).astype(np.float32)
    t = lambda a, dt=torch.float32: torch.tensor(a, device=DEV, dtype=dt)
    dS, dc = t(S), [t(c) for c in caches]
    dcw, donw = [t(w) for w in cw], t(onw)
    S_ref, c_ref = S.astype(np.float64), [c.astype(np.float64) for c in caches]
    to4 = lambda x, n, dd: x.reshape(B, 1, n, dd).permute(0, 2, 1, 3)
    for step in range(3):
        qr, kr, vr = f(B, 1, kd), f(B, 1, kd), f(B, 1, vd)
        g = -rng.uniform(0.0, 1.0, (B, 1, kd)).astype(np.float32)
        b = rng.uniform(0.0, 1.0, (B, 1, kd)).astype(np.float32)
        w = rng.uniform(0.0, 1.0, (B, 1, vd)).astype(np.float32)
        gate = f(B, 1, vd)
        dq, dk, dv, db, dw, dgate = (t(x, dtype) for x in (qr, kr, vr, b, w, gate))
        dg = t(g)
        out = torch.empty(B, 1, HV, V, device=DEV, dtype=dtype)
        a = ops.recurrent_args(to4(dq, H, K), to4(dk, H, K), to4(dv, HV, V), to4(dg, H, K), to4(db, H, K),
                               to4(dw, HV, V), dS, out.permute(0, 2, 1, 3), K ** -0.5, num_heads=H, grouped=True,
                               prologue=1, conv_w=dcw, conv_in=dc, conv_out=dc, gate=to4(dgate, HV, V),
                               o_norm_weight=donw, norm_eps=1e-5)
        bg._lib.check(bg.LIB.gdn2_recurrent_fwd(ctypes.byref(a), ops.stream_handle()))
        torch.cuda.synchronize()
        r = lambda x: x.float().cpu().numpy().astype(np.float64)
        acts, new_c = [], []
        for i, x in enumerate((dq, dk, dv)):
            y, nc = O.short_conv_1d(r(x), cw[i].astype(np.float64), c_ref[i])
            acts.append(y)
            new_c.append(nc)
        q4 = O.l2_normalize_4d(acts[0].reshape(B, 1, H, K).transpose(0, 2, 1, 3), 1e-6)
        k4 = O.l2_normalize_4d(acts[1].reshape(B, 1, H, K).transpose(0, 2, 1, 3), 1e-6)
        v4 = acts[2].reshape(B, 1, HV, V).transpose(0, 2, 1, 3)
        tr = lambda x, n, dd: r(x).reshape(B, 1, n, dd).transpose(0, 2, 1, 3)
        o_ref, S_ref = O.fused_recurrent_forward(q4, k4, v4, tr(dg, H, K), tr(db, H, K), tr(dw, HV, V), S_ref,
                                                 K ** -0.5)
        y_ref = O.rms_norm_gate_per_head(o_ref.transpose(0, 2, 1, 3), r(dgate).reshape(B, 1, HV, V),
                                         onw.astype(np.float64), 1e-5)
        c_ref = new_c
        _check(out.float().cpu().numpy(), y_ref, dtype, f"step {step} out")
        assert_close(dS.cpu().numpy(), S_ref, what=f"step {step} state", **F32_TOL)
        for i in range(3):
            assert_close(dc[i].cpu().numpy(), c_ref[i], what=f"step {step} cache {i}", rtol=0, atol=0)
    assert bg._lib.read_device_errors() == 0
