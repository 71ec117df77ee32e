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


@pytest.mark.parametrize("L", [64, 200, 1000])
def test_tcgen05_chunk_scan_matches_mma_sync_kernel(L):
    """The tcgen05 chunk scan against the mma.sync kernel and the fp32 oracle."""
    from sigma0_b200.ops._ext import ext
    import test_gpu_mamba3 as T
    C = ext()
    m = T._layer(seed=5)
    B = 2
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    torch.manual_seed(L)
    proj = (torch.randn(B * L, ldp, device="cuda") * 0.5).to(torch.bfloat16)
    args = (proj, B, L, d.n_heads, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D,
            m.A_floor, 1e-6)
    C.m3_use_tc_scan(False)
    y0 = C.m3_fwd(*args)[0]
    C.m3_use_tc_scan(True)
    try:
        y1 = C.m3_fwd(*args)[0]
        torch.cuda.synchronize()
    finally:
        C.m3_use_tc_scan(False)
    assert C.m3_tc_error() == 0
    yr = T._oracle_y(m, proj[:, :d.d_in_proj].contiguous(), B, L)
    assert T.rel(y1, yr) < 2e-2, T.rel(y1, yr)
    assert T.rel(y1, y0) < 1e-2, T.rel(y1, y0)
