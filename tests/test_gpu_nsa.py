"""NSA's compressed and selected branches on the flash kernels (per-key position tables,
per-group query offsets, head-summed importance) against the tensor-expression path of
the same module on the same (bf16-rounded) values: outputs, importance and gradients."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("BS,SB,L,q_offset", [(32, 64, 700, 0), (26, 26, 300, 0), (32, 64, 20, 680)])
def test_nsa_branches_match_reference(BS, SB, L, q_offset):
    from sigma0_b200.models.nsa import NSABlock
    torch.manual_seed(BS + L)
    m = NSABlock(256, n_heads=4, block_size=BS, select_block=SB, block_counts=4).cuda()
    B, nh, hd = 2, m.nh, m.hd
    Lk = q_offset + L
    q = torch.randn(B, L, nh, hd, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Lk, nh, hd, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Lk, nh, hd, device="cuda").to(torch.bfloat16)
    scale = hd ** -0.5
    xs = [t.clone().requires_grad_(True) for t in (q, k, v)]
    ys = [t.float().clone().requires_grad_(True) for t in (q, k, v)]
    o1, imp1 = m._compressed(*xs, scale, q_offset)
    o2, imp2 = m._compressed(*ys, scale, q_offset)
    assert _rel(o1, o2) < 2e-2
    vis = imp2 > -1e8
    assert torch.equal(imp1 > -1e8, vis) and _rel(imp1[vis], imp2[vis]) < 2e-2
    s1 = m._select(*xs, imp2, scale, q_offset)          # same importance -> same block choice
    s2 = m._select(*ys, imp2, scale, q_offset)
    assert _rel(s1, s2) < 2e-2
    g = torch.randn(o2.shape, device="cuda")
    ((o1.float() * g).sum() + (s1.float() * g).sum()).backward()
    ((o2 * g).sum() + (s2 * g).sum()).backward()
    for name, a, b in zip("qkv", xs, ys):
        assert _rel(a.grad, b.grad) < 3e-2, (name, _rel(a.grad, b.grad))


def test_nsa_block_forward_backward_runs_kernels():
    from sigma0_b200.models.nsa import NSABlock
    from sigma0_b200.ops import _ext
    m = NSABlock(256, n_heads=4, block_size=32, select_block=64, block_counts=4, dtype=torch.bfloat16).cuda()
    _ext.reset_launch_count()
    m(torch.randn(2, 500, 256, device="cuda")).sum().backward()
    assert _ext.launch_count() >= 4


@pytest.mark.parametrize("hd", [64, 128])
def test_block_indirect_attention_matches_the_gathered_blocks(hd):
    """Query groups over selected 64-key blocks read in place (``flash_attention_blocks``)
    against the same attention over a gathered copy of the blocks: outputs and q / k / v
    gradients, with blocks shared between groups (their key gradients add up)."""
    from sigma0_b200.ops.attention import flash_attention, flash_attention_blocks
    torch.manual_seed(hd)
    B, nblk, nh, ng, S = 2, 10, 2, 5, 4
    Lsrc, E = nblk * 64, B * ng
    k = torch.randn(B, Lsrc, nh, hd, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Lsrc, nh, hd, device="cuda").to(torch.bfloat16)
    q = torch.randn(E, 64, nh, hd, device="cuda").to(torch.bfloat16)
    top = torch.stack([torch.randperm(nblk)[:S] for _ in range(E)]).cuda()
    off = torch.arange(S * 64, device="cuda")
    kpos = top[:, off // 64] * 64 + off % 64
    qoff = (256 + torch.arange(ng, device="cuda") * 64).repeat(B)
    scale = hd ** -0.5
    xs = [t.clone().requires_grad_(True) for t in (q, k, v)]
    o1 = flash_attention_blocks(xs[0], xs[1], xs[2], top, kpos, qoff, scale)
    ys = [t.clone().requires_grad_(True) for t in (q, k, v)]
    src = torch.arange(E, device="cuda") // ng
    ksel = ys[1].reshape(B, nblk, 64, nh, hd)[src[:, None], top].reshape(E, S * 64, nh, hd)
    vsel = ys[2].reshape(B, nblk, 64, nh, hd)[src[:, None], top].reshape(E, S * 64, nh, hd)
    o2 = flash_attention(ys[0], ksel, vsel, scale=scale, kpos=kpos, qoff=qoff)
    assert _rel(o1, o2) < 1e-2, _rel(o1, o2)
    g = torch.randn(o2.shape, device="cuda")
    (o1.float() * g).sum().backward()
    (o2.float() * g).sum().backward()
    for name, a, b in zip("qkv", xs, ys):
        assert _rel(a.grad, b.grad) < 2e-2, (name, _rel(a.grad, b.grad))
