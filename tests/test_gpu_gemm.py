"""The tcgen05 GEMM (``csrc/gemm_tc.cu``) against an fp32 torch reference of the same product."""
import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


@cuda
@pytest.mark.parametrize("M,K,N", [(256, 128, 256), (1000, 200, 296), (4096, 1024, 4384), (129, 72, 520)])
def test_mm_forward(M, K, N):
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    y = gemm.mm(x, w)
    ref = x.float() @ w.float()
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    assert _rel(y, ref) < 8e-3
    assert gemm.status(x) == 0


@cuda
@pytest.mark.parametrize("M,K,N", [(256, 256, 128), (1000, 296, 200), (4096, 4384, 1024)])
def test_mm_input_gradient(M, K, N):
    """dy [M, N] @ W[K, N]^T."""
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(1)
    dy = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    w = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    y = gemm.mm_nt(dy, w)
    assert _rel(y, dy.float() @ w.float().t()) < 8e-3


@cuda
@pytest.mark.parametrize("T,M,N,split", [(512, 128, 256, 1), (3000, 200, 296, 0), (8192, 1024, 4384, 0),
                                         (8192, 1024, 1024, 3)])
def test_weight_gradient_accumulates_in_fp32(T, M, N, split):
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(T, M, device="cuda", generator=g).bfloat16()
    dy = torch.randn(T, N, device="cuda", generator=g).bfloat16()
    out = torch.randn(M, N, device="cuda", generator=g)
    before = out.clone()
    gemm.mm_tn_acc(x, dy, out, split_k=split)
    ref = before + x.float().t() @ dy.float()
    assert _rel(out, ref) < 2e-5 * (T ** 0.5) + 1e-5
    assert gemm.status(x) == 0


@cuda
def test_weight_gradient_into_a_smaller_view():
    """The output may be the leading block of the product (padded projection columns dropped)
    and a strided view of a larger buffer."""
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(700, 264, device="cuda", generator=g).bfloat16()
    dy = torch.randn(700, 520, device="cuda", generator=g).bfloat16()
    big = torch.zeros(300, 600, device="cuda")
    view = big[:256, :516]
    gemm.mm_tn_acc(x, dy, view)
    ref = (x.float().t() @ dy.float())[:256, :516]
    assert _rel(view, ref) < 1e-5
    assert float(big[256:].abs().max()) == 0.0 and float(big[:, 516:].abs().max()) == 0.0


@cuda
def test_strided_operands():
    """Row-strided operands (a slice of a wider buffer) are read in place."""
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(4)
    buf = torch.randn(512, 400, device="cuda", generator=g).bfloat16()
    x = buf[:, 8:264]                        # [512, 256], row stride 400
    w = torch.randn(256, 384, device="cuda", generator=g).bfloat16()
    assert _rel(gemm.mm(x, w), x.float() @ w.float()) < 8e-3
