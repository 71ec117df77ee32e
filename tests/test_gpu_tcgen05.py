"""The tcgen05 building blocks (descriptors, TMEM layout) against torch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N", [64, 128])
@pytest.mark.parametrize("K", [64, 128])
def test_tcgen05_gemm_m128(N, K):
    from sigma0_b200.ops._ext import ext
    torch.manual_seed(N + K)
    A = torch.randn(128, K, device="cuda").to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    D, err = ext().tc_gemm_test(A, B, 128)
    torch.cuda.synchronize()
    assert int(err) == 0
    ref = A.float() @ B.float().t()
    assert torch.allclose(D, ref, atol=1e-3, rtol=1e-4), (D - ref).abs().max()
