"""Context-parallel GDN / KDA mixer on CPU ranks (gloo, worlds 2 and 3) against the
full-sequence mixer: each rank's output segment, its input gradient and the parameter
gradients summed over the group; plus the segment-transition identity it rests on."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rel(a, b):
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _mixer(kda, conv=True):
    from sigma0_b200.models.gdn import GDN
    torch.manual_seed(0)
    m = GDN(64, num_heads=4, head_dim=16, expand_v=2, chunk_size=16, use_kda=kda, use_conv=conv)
    with torch.no_grad():
        m.out_norm.scale.normal_(1.0, 0.3)
        m.gk_proj.bias.fill_(2.0)
    return m


def _data(L):
    g = torch.Generator().manual_seed(1)
    return torch.randn(2, L, 64, generator=g), torch.randn(2, L, 64, generator=g)


def _worker(rank, world, port, kda, L, out, conv=True):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        torch.set_num_threads(1)
        from sigma0_b200.parallel.cp import split_sequence
        from sigma0_b200.parallel.cp_gdn import GDNCP
        full = _mixer(kda, conv)
        m = GDNCP(full)
        x, gout = _data(L)
        xs = split_sequence(x).clone().requires_grad_(True)
        y = m(xs)
        (y * split_sequence(gout)).sum().backward()
        grads = {n: p.grad.clone() for n, p in full.named_parameters() if p.grad is not None}
        for g in grads.values():
            dist.all_reduce(g)
        torch.save({"y": y.detach(), "dx": xs.grad, "grads": grads}, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


def test_segment_transition_identity():
    from sigma0_b200.models.gdn import gated_delta_chunked, l2_normalize
    torch.manual_seed(0)
    B, L, nh, hd, hvd = 2, 150, 2, 16, 32
    q = l2_normalize(torch.randn(B, L, nh, hd)) * hd ** -0.5
    k, v = l2_normalize(torch.randn(B, L, nh, hd)), torch.randn(B, L, nh, hvd)
    beta = torch.sigmoid(torch.randn(B, L, nh))
    for kda in (False, True):
        alog = torch.nn.functional.logsigmoid(torch.randn(B, L, nh, hd if kda else 1) + 2)
        S0 = torch.randn(B, nh, hvd, hd)
        _, S_zero, T = gated_delta_chunked(q, k, v, beta, alog, 16, return_transition=True)
        _, S_full = gated_delta_chunked(q, k, v, beta, alog, 16, S0=S0)
        assert _rel(S_full, S0 @ T + S_zero) < 1e-6


@pytest.mark.parametrize("kda,world,L,conv", [(False, 2, 80, True), (True, 2, 80, True), (False, 3, 90, True),
                                             (True, 2, 64, False)])
def test_context_parallel_gdn_matches_full(kda, world, L, conv, tmp_path):
    full = _mixer(kda, conv)
    x, gout = _data(L)
    x.requires_grad_(True)
    y = full(x)
    (y * gout).sum().backward()
    out = str(tmp_path / "r")
    mp.spawn(_worker, args=(world, _port(), kda, L, out, conv), nprocs=world, join=True)
    res = [torch.load(f"{out}.{r}") for r in range(world)]
    Ls = L // world
    for r, part in enumerate(res):
        sl = slice(Ls * r, Ls * (r + 1))
        assert _rel(part["y"], y.detach()[:, sl]) < 2e-5, (r, _rel(part["y"], y.detach()[:, sl]))
        assert _rel(part["dx"], x.grad[:, sl]) < 2e-5, (r, _rel(part["dx"], x.grad[:, sl]))
    for n, p in full.named_parameters():
        if p.grad is not None:
            err = (res[0]["grads"][n] - p.grad).norm().item()
            assert err <= 5e-5 * p.grad.norm().item() + 1e-5, (n, err)
