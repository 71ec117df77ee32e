"""Tensor parallelism inside the Trainer on gloo CPU ranks: ``Trainer(tp=2)`` (heads split
over two ranks) and ``Trainer(tp=2)`` on four ranks (a 2 x 2 dp x tp mesh) train to the same
losses as the single-process trainer on the same data; the global gradient norm counts
each head slice once and each replicated parameter once."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _args(arch):
    from sigma0_b200.models import preset_args
    extra = dict(gdn_head_dim=16) if arch == "gdn" else dict(mamba3_d_state=16, mamba3_headdim=16)
    return preset_args("smoke", architecture=arch, d_model=64, n_messages=4, micro_bsz=2, warmup_end=0.0,
                       ssm_lr_base=3e-3, max_grad_norm=0.05, **extra)


def _batch(n, seed=0):
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    days = make_sequences(n, 5, seed=seed)
    ds = LobWindowDataset.from_days(days, 4, token_mode="22tok")
    return collate([ds[i] for i in range(n)])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _losses(tr, tok, lab, book, steps=3):
    return [float(tr.step_device(tok, lab, book)) for _ in range(steps)]


def _worker(rank, world, port, arch, tp, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.train.trainer import Trainer
        torch.set_num_threads(1)
        tr = Trainer(_args(arch), device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=0, tp=tp)
        tok, lab, book = _batch(4)
        per = tok.shape[0] // tr.world                  # the batch is split over the dp axis only
        sl = slice(tr.rank * per, (tr.rank + 1) * per)
        ls = _losses(tr, tok[sl], lab[sl], book[sl])
        t = torch.tensor(ls)
        dist.all_reduce(t)                              # mean over every rank = mean over dp groups
        if rank == 0:
            torch.save(t / world, out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("arch,world", [("gdn", 2), ("mamba3", 2), ("gdn", 4)])
def test_tp_trainer_matches_single_process(arch, world, tmp_path):
    from sigma0_b200.train.trainer import Trainer
    out = str(tmp_path / "l.pt")
    mp.spawn(_worker, args=(world, _free_port(), arch, 2, out), nprocs=world, join=True)
    got = torch.load(out)
    tok, lab, book = _batch(4)
    # with two dp groups each sees half of the batch; the single process sees all of it, whose
    # loss is the mean of the halves' losses (equal sizes) and whose gradient is their average
    tr = Trainer(_args(arch), device=torch.device("cpu"), total_steps=10, seed=0)
    ref = torch.tensor(_losses(tr, tok, lab, book))
    assert torch.allclose(got, ref, rtol=2e-4, atol=2e-4), (got, ref)


def _hier_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.train.trainer import Trainer
        torch.set_num_threads(1)
        res = {}
        for hier in (False, True):
            tr = Trainer(_args("mamba3"), device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=0,
                         hierarchical=hier, gpus_per_node=2)
            tok, lab, book = _batch(4)
            sl = slice(rank, rank + 1)
            _losses(tr, tok[sl], lab[sl], book[sl])
            res[hier] = tr.opt.flat.clone()
        if rank == 0:
            torch.save(res, out)
    finally:
        dist.destroy_process_group()


def test_hierarchical_step_matches_flat_data_parallel(tmp_path):
    """Four ranks as 2 nodes x 2 GPUs: reduce-scatter in the node, all-reduce across nodes,
    all-gather -- the same parameters as the flat all-reduce."""
    out = str(tmp_path / "h.pt")
    mp.spawn(_hier_worker, args=(4, _free_port(), out), nprocs=4, join=True)
    r = torch.load(out)
    n = min(r[False].numel(), r[True].numel())
    assert torch.allclose(r[False][:n], r[True][:n], rtol=1e-5, atol=1e-6)
