"""Context-parallel S5 layer on CPU ranks (gloo, worlds 2 and 3) against the full-sequence
layer: each rank's output segment, its input gradient and the parameter gradients summed
over the group."""
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


def _layer():
    from sigma0_b200.models.s5 import make_s5_factory
    torch.manual_seed(0)
    return make_s5_factory(32, 2)(24)


def _data(L):
    g = torch.Generator().manual_seed(1)
    return torch.randn(2, L, 24, generator=g), torch.randn(2, L, 24, generator=g)


def _worker(rank, world, port, L, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        torch.set_num_threads(1)
        from sigma0_b200.parallel.cp_s5 import S5CP
        m = S5CP(_layer())
        u, gout = _data(L)
        Ls = L // world
        seg = u[:, rank * Ls:(rank + 1) * Ls].clone().requires_grad_(True)
        y = m(seg)
        (y * gout[:, rank * Ls:(rank + 1) * Ls]).sum().backward()
        torch.save({"y": y.detach(), "du": seg.grad, "grads": {n: p.grad for n, p in m.inner.named_parameters()}},
                   f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_s5_context_parallel_matches_full(world, tmp_path):
    L = 36
    full = _layer()
    u, gout = _data(L)
    u.requires_grad_(True)
    y = full(u)
    (y * gout).sum().backward()
    out = str(tmp_path / "r")
    mp.spawn(_worker, args=(world, _port(), L, out), nprocs=world, join=True)
    res = [torch.load(f"{out}.{r}") for r in range(world)]
    Ls = L // world
    for r, d in enumerate(res):
        ref_y, ref_du = y[:, r * Ls:(r + 1) * Ls].detach(), u.grad[:, r * Ls:(r + 1) * Ls]
        assert (d["y"] - ref_y).norm() <= 2e-5 * ref_y.norm(), r
        assert (d["du"] - ref_du).norm() <= 2e-5 * ref_du.norm(), r
    for n, p in full.named_parameters():
        g = sum(d["grads"][n] for d in res)
        err = (g - p.grad).norm().item()
        assert err <= 5e-5 * p.grad.norm().item() + 1e-6, (n, err)


def test_bidirectional_layer_is_refused():
    from sigma0_b200.models.s5 import make_s5_factory
    from sigma0_b200.parallel.cp_s5 import S5CP
    with pytest.raises(ValueError):
        S5CP(make_s5_factory(32, 2, bidirectional=True)(24))
