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


@cuda
def test_trainer_gradients_match_the_library_gemm_arm():
    """One training step of a small CUDA Mamba3 LOB model: the flat gradient with the tcgen05
    projections (weight gradients reduce-added straight into the optimizer's buffer) equals the
    one computed with torch.matmul."""
    from sigma0_b200.data import LobWindowDataset, collate, make_sequences
    from sigma0_b200.models import preset_args
    from sigma0_b200.ops import gemm
    from sigma0_b200.train.trainer import Trainer
    args = preset_args("smoke", impl="cuda", d_model=256, mamba3_d_state=128, mamba3_headdim=64, n_messages=24,
                       micro_bsz=2, n_layers=2, dtype="bfloat16")
    days = make_sequences(2, args.n_messages + 1, seed=5)
    ds = LobWindowDataset.from_days(days, args.n_messages, token_mode=args.token_mode)
    batch = [t.cuda() for t in collate([ds[i] for i in range(2)])]
    grads = []
    saved = gemm.USE_TC
    try:
        for tc in (True, False):
            gemm.USE_TC = tc
            tr = Trainer(args, device=torch.device("cuda"), world=1, rank=0, total_steps=10, seed=0)
            tr.opt.zero_grad()
            loss, _ = tr.model.loss(batch[0], batch[2], batch[1])
            loss.backward()
            grads.append(tr.opt.grad.clone())
    finally:
        gemm.USE_TC = saved
    assert torch.isfinite(grads[0]).all() and float(grads[0].abs().sum()) > 0
    assert _rel(grads[0], grads[1]) < 2e-2


@cuda
def test_weight_gradient_of_an_odd_width_parameter():
    """A 503-column weight (the book layers): the fp32 result rows are padded for the tensor
    map and the leading block comes back."""
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(6)
    p = torch.nn.Parameter(torch.zeros(960, 503, device="cuda"))
    x = torch.randn(2000, 960, device="cuda", generator=g).bfloat16()
    dy = torch.randn(2000, 504, device="cuda", generator=g).bfloat16()
    got = gemm.wgrad(p, x, dy)
    assert got.shape == (960, 503)
    assert _rel(got, (x.float().t() @ dy.float())[:, :503]) < 1e-5


@cuda
def test_fused_gelu_forward_epilogue():
    import torch.nn.functional as F
    from sigma0_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.randn(3000, 512, device="cuda", generator=g) * 0.1).bfloat16()
    w = (torch.randn(512, 1024, device="cuda", generator=g) * 0.1).bfloat16()
    o, gl = gemm.proj_gelu(x, w)
    ref = x.float() @ w.float()
    assert _rel(o, ref) < 8e-3
    # g is the GELU of the stored bf16 o
    assert _rel(gl, F.gelu(o.float(), approximate="tanh")) < 8e-3
