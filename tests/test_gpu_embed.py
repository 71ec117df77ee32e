"""The embedding gather kernels (csrc/embed.cu) against torch: the token embedding and the
1-token model's 24-field embedding sum, forward and scatter-add backward."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nf,D", [(1, 1024), (24, 64), (24, 1028)])
def test_embed_sum_matches_torch(nf, D):
    from sigma0_b200.models.common import embed_sum
    g = torch.Generator(device="cuda").manual_seed(nf)
    rows = [int(torch.randint(5, 300, (1,)).item()) for _ in range(nf)]
    tabs = [torch.randn(r, D, device="cuda", generator=g).requires_grad_(True) for r in rows]
    idx = torch.stack([torch.randint(0, r, (3, 700), device="cuda", generator=g) for r in rows], -1)
    out = embed_sum(idx, tabs)
    ref = sum(t.detach()[idx[..., f]] for f, t in enumerate(tabs))
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-5)
    go = torch.randn_like(out)
    (out * go).sum().backward()
    for f, t in enumerate(tabs):
        want = torch.zeros_like(t).index_add_(0, idx[..., f].reshape(-1), go.reshape(-1, D))
        assert torch.allclose(t.grad, want, rtol=1e-4, atol=1e-4), f


def test_one_token_model_on_cuda_matches_torch_path():
    from sigma0_b200.models import preset_args, build_model
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    args = dict(token_mode="1tok", d_model=256, mamba3_d_state=128, mamba3_headdim=64, n_messages=20, micro_bsz=2,
                n_layers=1, dtype="bfloat16")
    torch.manual_seed(0)
    mc = build_model(preset_args("smoke", impl="cuda", **args)).cuda()
    mt = build_model(preset_args("smoke", impl="torch", **args)).cuda()
    mt.load_state_dict(mc.state_dict())
    ds = LobWindowDataset.from_days(make_sequences(2, 21, seed=1), 20, token_mode="1tok")
    x, y, book = (t.cuda() for t in collate([ds[0], ds[1]]))
    lc, _ = mc.loss(x, book.float(), y)
    lt, _ = mt.loss(x, book.float(), y)
    lc.backward()
    lt.backward()
    assert abs(lc.item() - lt.item()) < 2e-2 * abs(lt.item())
    for (n, a), (_, b) in zip(mc.named_parameters(), mt.named_parameters()):
        if a.grad is None and b.grad is None:
            continue
        err = ((a.grad - b.grad).norm() / (b.grad.norm() + 1e-12)).item()
        assert err < 6e-2, (n, err)
