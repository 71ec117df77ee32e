"""Data-parallel training on CPU ranks (gloo): replicated and sharded (ZeRO) updates,
bf16 gradient wire, gradient accumulation, and sharded checkpoints restored at a
different world size."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _args():
    from sigma0_b200.models import preset_args
    return preset_args("smoke", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_messages=4, micro_bsz=2,
                       warmup_end=0.0, ssm_lr_base=3e-3)


def _batch(n=4, seed=0):
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


def _worker(rank, world, port, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.train.trainer import Trainer
        torch.set_num_threads(1)
        tr = Trainer(_args(), device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=0,
                     sharded=mode.startswith("sharded"), grad_wire_dtype="bfloat16" if "bf16" in mode else "float32")
        tok, lab, book = _batch()
        per = tok.shape[0] // world
        sl = slice(rank * per, (rank + 1) * per)
        for _ in range(3):
            tr.step_device(tok[sl], lab[sl], book[sl])
        if mode == "sharded_ckpt":
            from sigma0_b200.ckpt import CheckpointManager
            mgr = CheckpointManager(os.path.join(out_dir, "ck"), rank=rank, world=world, barrier=dist.barrier)
            mgr.save(3, tr, config={"mode": mode})
            torch.save({"m": tr.opt.m.clone(), "lo": tr.opt.lo}, os.path.join(out_dir, f"m{rank}.pt"))
        if rank == 0:
            torch.save(tr.opt.flat.clone(), os.path.join(out_dir, "flat.pt"))
    finally:
        dist.destroy_process_group()


def _run(world, mode, tmp_path):
    mp.spawn(_worker, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world, join=True)
    return torch.load(os.path.join(tmp_path, "flat.pt"))


def _single(accum=1):
    from sigma0_b200.train.trainer import Trainer
    tr = Trainer(_args(), device=torch.device("cpu"), total_steps=10, seed=0, accum_steps=accum)
    tok, lab, book = _batch()
    for _ in range(3):
        tr.step_device(tok, lab, book)
    return tr


def test_replicated_dp_matches_single_process(tmp_path):
    ref = _single().opt.flat
    got = _run(2, "replicated", tmp_path)
    n = ref.numel()
    assert torch.allclose(got[:n], ref, atol=2e-5, rtol=1e-4), (got[:n] - ref).abs().max()


def test_sharded_dp_matches_single_process(tmp_path):
    ref = _single().opt.flat
    got = _run(2, "sharded", tmp_path)
    n = ref.numel()
    assert torch.allclose(got[:n], ref, atol=2e-5, rtol=1e-4), (got[:n] - ref).abs().max()


def test_bf16_wire_close(tmp_path):
    ref = _single().opt.flat
    got = _run(2, "replicated_bf16", tmp_path)
    n = ref.numel()
    assert (got[:n] - ref).abs().max() < 5e-3


def test_grad_accumulation_matches_full_batch():
    a = _single(1).opt.flat
    b = _single(2).opt.flat
    assert torch.allclose(a, b, atol=2e-5, rtol=1e-4), (a - b).abs().max()


def test_sharded_checkpoint_restores_at_world_one(tmp_path):
    from sigma0_b200.ckpt import CheckpointManager
    from sigma0_b200.train.trainer import Trainer
    _run(2, "sharded_ckpt", tmp_path)
    tr = Trainer(_args(), device=torch.device("cpu"), total_steps=10, seed=1)
    meta = CheckpointManager(os.path.join(tmp_path, "ck")).restore(tr)
    assert meta["restored_step"] == 3 and tr.opt.step_count == 3
    assert tr.step_idx == 6   # elastic remap: global batch 4 at world 2 -> 2 at world 1
    flat = torch.load(os.path.join(tmp_path, "flat.pt"))
    assert torch.equal(tr.opt.flat, flat[:tr.opt.numel])
    for r in range(2):
        d = torch.load(os.path.join(tmp_path, f"m{r}.pt"))
        lo = d["lo"]
        k = min(d["m"].numel(), tr.opt.numel - lo)
        assert torch.equal(tr.opt.m[lo:lo + k], d["m"][:k])


def _diloco_worker(rank, world, port, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.train.trainer import Trainer
        from sigma0_b200.train.diloco import DiLoCo
        torch.set_num_threads(1)
        tr = Trainer(_args(), device=torch.device("cpu"), world=1, rank=0, total_steps=10, seed=0)
        dl = DiLoCo(tr, inner_steps=2, mode=mode)
        tok, lab, book = _batch()
        per = tok.shape[0] // world
        sl = slice(rank * per, (rank + 1) * per)
        for _ in range(4):
            dl.step(tok[sl], lab[sl], book[sl])
        torch.save({"flat": tr.opt.flat.clone(), "outer": dl.outer_steps}, os.path.join(out_dir, f"d{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["diloco", "fedavg"])
def test_diloco_ranks_agree_after_outer_steps(tmp_path, mode):
    mp.spawn(_diloco_worker, args=(2, _free_port(), mode, str(tmp_path)), nprocs=2, join=True)
    a, b = (torch.load(os.path.join(tmp_path, f"d{r}.pt")) for r in range(2))
    assert a["outer"] == 2 and torch.equal(a["flat"], b["flat"])
    assert torch.isfinite(a["flat"]).all()


def test_fedavg_one_inner_step_is_parameter_average(tmp_path):
    """FedAvg with H=1 on a single process equals the local step (average of one)."""
    from sigma0_b200.train.trainer import Trainer
    from sigma0_b200.train.diloco import DiLoCo
    tr = Trainer(_args(), device=torch.device("cpu"), total_steps=10, seed=0)
    ref = Trainer(_args(), device=torch.device("cpu"), total_steps=10, seed=0)
    dl = DiLoCo(tr, inner_steps=1, mode="fedavg")
    tok, lab, book = _batch()
    dl.step(tok, lab, book)
    ref.step_device(tok, lab, book)
    assert torch.allclose(tr.opt.flat, ref.opt.flat, atol=1e-7)


def _cp_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.train.trainer import Trainer
        torch.set_num_threads(1)
        tr = Trainer(_args(), device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=0,
                     context_parallel=True)
        tok, lab, book = _batch()
        losses = [float(tr.step_device(tok, lab, book)) for _ in range(3)]
        if rank == 0:
            torch.save({"flat": tr.opt.flat.clone(), "losses": losses}, os.path.join(out_dir, "cp.pt"))
    finally:
        dist.destroy_process_group()


def test_context_parallel_trainer_matches_single_process(tmp_path):
    """Two context-parallel ranks, each holding half of every sequence, take the same three
    optimizer steps as one process on the whole sequences."""
    from sigma0_b200.train.trainer import Trainer
    torch.set_num_threads(2)
    tr = Trainer(_args(), device=torch.device("cpu"), world=1, rank=0, total_steps=10, seed=0)
    tok, lab, book = _batch()
    ref_losses = [float(tr.step_device(tok, lab, book)) for _ in range(3)]
    mp.spawn(_cp_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    res = torch.load(os.path.join(str(tmp_path), "cp.pt"))
    np.testing.assert_allclose(res["losses"], ref_losses, rtol=2e-5)
    d = (res["flat"] - tr.opt.flat).norm() / tr.opt.flat.norm()
    assert d < 1e-5, float(d)
