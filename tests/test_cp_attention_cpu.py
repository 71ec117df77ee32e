"""Context-parallel transformer and NSA blocks on CPU ranks (gloo, world 2) against the
full-sequence blocks: each rank's output segment, its input gradient, and the parameter
gradients summed over the group."""
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


def _block(kind):
    torch.manual_seed(0)
    if kind == "transformer":
        from sigma0_b200.models.transformer import TransformerBlock
        return TransformerBlock(64, n_heads=4, d_ff=128)
    from sigma0_b200.models.nsa import NSABlock
    return NSABlock(64, n_heads=4, block_size=8, select_block=16, block_counts=2, window_size=20,
                    full_causal_window=kind == "nsa")


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randn(2, 64, 64, generator=g), torch.randn(2, 64, 64, generator=g)


def _worker(rank, world, port, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        torch.set_num_threads(1)
        from sigma0_b200.parallel.cp import split_sequence
        from sigma0_b200.parallel.cp_attention import NSABlockCP, TransformerBlockCP
        full = _block(kind)
        m = TransformerBlockCP(full) if kind == "transformer" else NSABlockCP(full)
        x, gout = _data()
        xs = split_sequence(x).clone().requires_grad_(True)
        y = m(xs)
        (y * split_sequence(gout)).sum().backward()
        grads = {n: p.grad.clone() for n, p in full.named_parameters() if p.grad is not None}
        for g in grads.values():
            dist.all_reduce(g)
        torch.save({"y": y.detach(), "dx": xs.grad, "grads": grads}, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["transformer", "nsa", "nsa_window"])
def test_context_parallel_attention_matches_full(kind, tmp_path):
    full = _block(kind)
    x, gout = _data()
    x.requires_grad_(True)
    y = full(x)
    (y * gout).sum().backward()
    out = str(tmp_path / "r")
    mp.spawn(_worker, args=(2, _port(), kind, out), nprocs=2, join=True)
    res = [torch.load(f"{out}.{r}") for r in range(2)]
    for r, part in enumerate(res):
        sl = slice(32 * r, 32 * (r + 1))
        assert _rel(part["y"], y.detach()[:, sl]) < 2e-5
        assert _rel(part["dx"], x.grad[:, sl]) < 2e-5
    for n, p in full.named_parameters():
        if p.grad is not None:
            # relative, plus an absolute floor: some gradients are zero in exact arithmetic
            # (a key bias shifts every score of a row equally and cancels in the softmax)
            err = (res[0]["grads"][n] - p.grad).norm().item()
            assert err <= 5e-5 * p.grad.norm().item() + 1e-5, (kind, n, err)


def test_shard_model_cp_wraps_every_sequence_mixer():
    from sigma0_b200.models.mamba3 import Mamba3
    from sigma0_b200.models.nsa import NSABlock
    from sigma0_b200.models.transformer import TransformerBlock
    from sigma0_b200.parallel.cp import Mamba3CP, shard_model_cp
    from sigma0_b200.parallel.cp_attention import NSABlockCP, TransformerBlockCP
    from sigma0_b200.models.gdn import GDN
    from sigma0_b200.parallel.cp_gdn import GDNCP
    from sigma0_b200.models.s5 import make_s5_factory
    from sigma0_b200.parallel.cp_s5 import S5CP
    m = torch.nn.Sequential(Mamba3(64, d_state=16, headdim=16, chunk_size=16), TransformerBlock(64, n_heads=4),
                            NSABlock(64, n_heads=4, block_size=8, select_block=16), GDN(64, num_heads=4, head_dim=16),
                            make_s5_factory(32, 2)(64))
    shard_model_cp(m)
    assert [type(c) for c in m] == [Mamba3CP, TransformerBlockCP, NSABlockCP, GDNCP, S5CP]
