"""gdn2_chunk_fwd_noalloc (static device scratch, no allocation) against
gdn2_chunk_fwd (caller workspace), both called through the C ABI.

Two calls in a row share the one scratch array: the second, smaller call
runs over what the first left behind, and must still match.  Both entry
points run the same kernels on the same inputs, so the results agree to
the f32 tolerance for f32 inputs and to the bf16 criterion for bf16.
The file name sorts last so the test also runs after every other GPU test.
"""
import ctypes

import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import F32_TOL, assert_close, assert_close_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(B, HV, T, K, V, dtype, seed, epilogue):
    arrs = O.make_core_inputs(B, HV, T, K, V, seed=seed, dtype=np.float32)
    d = {k: torch.tensor(arrs[k], dtype=torch.float32 if k == "g" else dtype, device=DEV) for k in "qkvgbw"}
    rng = np.random.default_rng(seed + 1)
    d["s0"] = torch.tensor(rng.standard_normal((B, HV, K, V)).astype(np.float32), device=DEV)
    if epilogue:
        d["gate"] = torch.tensor(rng.standard_normal((B, HV, T, V)).astype(np.float32), dtype=dtype, device=DEV)
        d["onw"] = torch.tensor(rng.uniform(0.5, 1.5, V).astype(np.float32), device=DEV)
    return d


def _run(d, noalloc):
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    state = d["s0"].clone()
    out = torch.full_like(d["v"], float("nan"))
    K = d["q"].shape[-1]
    a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], state, out, K ** -0.5, 64,
                       gate=d.get("gate"), o_norm_weight=d.get("onw"), norm_eps=1e-5)
    s = ops.stream_handle()
    if noalloc:
        rc = bg.LIB.gdn2_chunk_fwd_noalloc(ctypes.byref(a), s)
    else:
        ws = ops.chunk_workspace(a, d["q"].device)
        rc = bg.LIB.gdn2_chunk_fwd(ctypes.byref(a), ops.ptr(ws), ws.numel(), s)
    bg._lib.check(rc)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), state.cpu().numpy()


def _compare(d, dtype, what):
    o_ref, s_ref = _run(d, noalloc=False)
    o, s = _run(d, noalloc=True)
    if dtype == torch.float32:
        assert_close(o, o_ref, what=f"{what} out", **F32_TOL)
        assert_close(s, s_ref, what=f"{what} state", **F32_TOL)
    else:
        assert_close_bf16(o, o_ref, what=f"{what} out")
        assert_close_bf16(s, s_ref, what=f"{what} state")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_two_calls(dtype):
    import burn_gdn2 as bg

    # bf16 with K = 128 runs the tensor-core kernels, f32 the CUDA-core ones
    K, V = (128, 128) if dtype == torch.bfloat16 else (64, 64)
    first = _case(2, 4, 300, K, V, dtype, seed=101, epilogue=True)
    second = _case(1, 3, 130, K, V, dtype, seed=202, epilogue=False)
    _compare(first, dtype, "call 1")
    _compare(second, dtype, "call 2")
    flags = ctypes.c_uint32(0)
    bg._lib.check(bg.LIB.gdn2_read_device_errors(ctypes.byref(flags)))
    assert flags.value == 0


def test_noalloc_rejects_oversized_call():
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    # 2 x 16 heads x 32 chunks of 64 tokens = 1024 records > the 448 that fit
    B, HV, T, K, V = 2, 16, 2048, 128, 128
    q = torch.zeros(B, HV, T, K, dtype=torch.bfloat16, device=DEV)
    g = torch.zeros(B, HV, T, K, device=DEV)
    v = torch.zeros(B, HV, T, V, dtype=torch.bfloat16, device=DEV)
    out = torch.full_like(v, 7.0)
    state = torch.zeros(B, HV, K, V, device=DEV)
    a = ops.chunk_args(q, q, v, g, q, v, state, out, K ** -0.5, 64)
    assert bg.LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a)) > 32 << 20
    rc = bg.LIB.gdn2_chunk_fwd_noalloc(ctypes.byref(a), ops.stream_handle())
    assert rc == 4  # GDN2_EWORKSPACE
    assert b"static array" in bg.LIB.gdn2_last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing launched
