"""GPU: the tcgen05 building blocks (shared-memory descriptors for K-major
and MN-major 128-byte-swizzled tiles, M = 64 and M = 128 TMEM accumulator
layouts) against a host matmul of the same bf16-rounded operands."""

import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = {0: (128, 64, 128), 1: (64, 32, 128), 2: (128, 64, 64), 3: (128, 128, 64)}


@pytest.mark.parametrize("test", sorted(CASES))
def test_umma_tile(test):
    import burn_gdn2 as bg
    from burn_gdn2 import ops

    M, N, K = CASES[test]
    g = torch.Generator(device="cuda").manual_seed(test)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    D = torch.full((M, N), float("nan"), device="cuda")
    bg._lib.check(bg.LIB.gdn2_selftest_umma(test, ops.ptr(A), ops.ptr(B), ops.ptr(D), ops.stream_handle()))
    torch.cuda.synchronize()
    assert bg._lib.read_device_errors() == 0
    ref = A.bfloat16().double() @ B.bfloat16().double()
    err = (D.double() - ref).abs().max().item()
    assert err < 1e-3 * ref.abs().max().item(), (test, err)
