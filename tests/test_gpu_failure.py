"""GPU: the failure path of the kernels' bounded waits, without a fault.
A wait that nothing completes gives up after its limit, sets the device
error bit that gdn2_read_device_errors reports, and the kernel returns; the
context stays usable for the next launch."""
import ctypes

import numpy as np
import pytest
import torch

import gdn2_oracle as O
from helpers import F32_TOL, assert_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    import burn_gdn2 as bg
    from burn_gdn2 import LIB, _lib

    torch.zeros(1, device="cuda")
    _lib.read_device_errors()  # start from a clear state
    done = ctypes.c_int32(-1)
    _lib.check(LIB.gdn2_selftest_wait(1000, 0, ctypes.byref(done)))  # nothing arrives: the wait runs out
    assert done.value == 0
    assert _lib.read_device_errors() & 1
    assert _lib.read_device_errors() == 0  # reading clears the bits
    _lib.check(LIB.gdn2_selftest_wait(1000, 1, ctypes.byref(done)))  # the phase completes
    assert done.value == 1
    assert _lib.read_device_errors() == 0

    # the context is still usable: a chunked forward afterwards matches the oracle
    B, HV, T, K, V = 1, 2, 70, 16, 16
    a = O.make_core_inputs(B, HV, T, K, V, seed=5, dtype=np.float32)
    d = {n: torch.tensor(a[n], device="cuda") for n in "qkvgbw"}
    o, s = bg.chunk_wy_forward(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"],
                               torch.zeros(B, HV, K, V, device="cuda"), K ** -0.5, 64)
    r = {n: a[n].astype(np.float64) for n in "qkvgbw"}
    o_ref, s_ref = O.chunk_wy_forward(r["q"], r["k"], r["v"], r["g"], r["b"], r["w"], np.zeros((B, HV, K, V)),
                                      K ** -0.5, 64)
    assert_close(o.cpu().numpy(), o_ref, what="out", **F32_TOL)
    assert_close(s.cpu().numpy(), s_ref, what="state", **F32_TOL)
