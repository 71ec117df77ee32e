"""The fused tensor-parallel GEMM + all-reduce kernel on one rank (plain buffers) against
torch: tcgen05 tiles, owner accumulation, bf16 conversion and the buffer reset between calls."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,K,N", [(128, 64, 128), (300, 512, 256), (1000, 256, 1024)])
def test_fused_row_parallel_single_rank(T, K, N):
    from sigma0_b200.parallel.tp_fused import FusedRowParallel
    torch.manual_seed(T + K + N)
    h = FusedRowParallel(max_rows=1024, n_out=N, device="cuda")
    for it in range(2):                                       # the accumulation buffer must come back zeroed
        y = torch.randn(T, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(K, N, device="cuda") / K ** 0.5).to(torch.bfloat16)
        out = h(y, w.t().contiguous())
        torch.cuda.synchronize()
        h.check()
        ref = y.float() @ w.float()
        err = ((out.float() - ref).norm() / ref.norm()).item()
        assert err < 1e-2, (it, err)


def test_fused_row_parallel_autograd():
    from sigma0_b200.parallel.tp_fused import FusedRowParallel, fused_row_parallel
    torch.manual_seed(0)
    h = FusedRowParallel(max_rows=256, n_out=128, device="cuda")
    y = torch.randn(200, 128, device="cuda", requires_grad=True)
    w = (torch.randn(128, 128, device="cuda") / 11).requires_grad_(True)
    out = fused_row_parallel(y, w, h)
    (out * torch.linspace(-1, 1, 128, device="cuda")).sum().backward()
    y2, w2 = y.detach().clone().requires_grad_(True), w.detach().clone().requires_grad_(True)
    ((y2 @ w2) * torch.linspace(-1, 1, 128, device="cuda")).sum().backward()
    assert ((out - (y2 @ w2)).norm() / (y2 @ w2).norm()).item() < 1e-2
    assert torch.allclose(y.grad, y2.grad, atol=1e-5) and torch.allclose(w.grad, w2.grad, atol=1e-4)
