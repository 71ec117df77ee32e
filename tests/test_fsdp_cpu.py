"""ZeRO-3 sharding of the fused layers' kernels (``parallel/fsdp.py``) on gloo CPU ranks:
the gathered kernels equal the unsharded ones, the reduce-scattered gradient shards equal
the sums over ranks, the sharded AdamW step equals AdamW on the full tensors, and a native
checkpoint of an FSDP trainer holds the full kernels."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    from sigma0_b200.models import preset_args
    from sigma0_b200.models.registry import build_model
    # impl "cuda" marks the layers as fused units; nothing runs here
    args = preset_args("smoke", impl="cuda", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_layers=2)
    torch.manual_seed(0)
    return build_model(args)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from sigma0_b200.ops import weights as W
        from sigma0_b200.parallel.fsdp import FSDP, fsdp_layers
        torch.set_num_threads(1)
        model = _model()
        layers = fsdp_layers(model)
        ref = {id(p): p.detach().clone() for l in layers for p in
               (l.seq.in_proj.kernel, l.seq.out_proj.kernel, l.out2.kernel)}
        fs = FSDP(model, world, rank, lr=1e-2, weight_decay=0.1)
        res = {"n_units": len(fs.units)}
        # 1. forward gathers reproduce the kernels (bf16 copies)
        ok = True
        for l in layers:
            fs.before_forward(l)
            for p in (l.seq.in_proj.kernel, l.seq.out_proj.kernel, l.out2.kernel):
                ok &= torch.equal(W.bf16(p).float(), ref[id(p)].bfloat16().float())
                ok &= p.data.stride() == (0, 0)          # no storage of its own at rest
        res["gather_ok"] = bool(ok)
        # 2. gradients: rank r writes (r + 1) * G; the shards hold the sum over ranks
        g = {}
        for l in reversed(layers):
            fs.before_backward(l)
            for p in (l.seq.in_proj.kernel, l.seq.out_proj.kernel, l.out2.kernel):
                gen = torch.Generator().manual_seed(p.numel())
                G = torch.randn(p.shape, generator=gen)
                g[id(p)] = G * sum(r + 1 for r in range(world))
                p.grad.add_(G * (rank + 1))
            fs.after_backward(l)
        fs.sync()
        full_g = {}
        for u in fs.units:
            shards = [torch.zeros_like(u.grad) for _ in range(world)]
            dist.all_gather(shards, u.grad)
            for k, p in enumerate(u.params):
                n, so = p.numel() // world, u.soffsets[k]           # row blocks, rank order = row order
                full_g[id(p)] = torch.cat([sh[so:so + n] for sh in shards]).view(p.shape)
        res["grad_ok"] = all(torch.allclose(full_g[k], g[k], rtol=1e-5, atol=1e-5) for k in g)
        # 3. one sharded AdamW step against the full-tensor update (averaged gradient)
        total = fs.grad_sumsq()
        fs.step(1.0, total, max_grad_norm=0.0)
        full = fs.full_parameters()
        b1, b2, eps, lr, wd = 0.9, 0.999, 1e-8, 1e-2, 0.1
        err = 0.0
        for u in fs.units:
            for p in u.params:
                G = g[id(p)] / world
                mm = (1 - b1) * G
                vv = (1 - b2) * G * G
                want = ref[id(p)] - lr * ((mm / (1 - b1)) / ((vv / (1 - b2)).sqrt() + eps) + wd * ref[id(p)])
                err = max(err, float((full[p] - want).abs().max()))
        res["step_err"] = err
        # 4. native checkpoint of an FSDP trainer: full kernels by Flax path, moment shards per rank
        from sigma0_b200.ckpt import CheckpointManager
        from sigma0_b200.models import preset_args
        from sigma0_b200.train.trainer import Trainer
        args = preset_args("smoke", impl="cuda", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_layers=2)
        tr = Trainer(args, device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=1, fsdp=True)
        for u in tr.fsdp.units:
            u.master.add_(0.5 * (rank + 1))
            u.m.fill_(rank + 1.0)
        want = tr.fsdp.full_parameters()
        mgr = CheckpointManager(os.path.dirname(out) + "/ck", rank=rank, world=world, barrier=dist.barrier)
        mgr.save(3, tr, blocking=True)
        tr2 = Trainer(args, device=torch.device("cpu"), world=world, rank=rank, total_steps=10, seed=2, fsdp=True)
        mgr.restore(tr2)
        got = tr2.fsdp.full_parameters()
        p1 = tr.fsdp.sharded_parameters()
        p2 = tr2.fsdp.sharded_parameters()
        res["ckpt_ok"] = all(torch.equal(want[a], got[b]) for a, b in zip(p1, p2)) and \
            all(torch.equal(u.m, torch.full_like(u.m, rank + 1.0)) for u in tr2.fsdp.units)
        if rank == 0:
            torch.save(res, out)
    finally:
        dist.destroy_process_group()


def test_fsdp_shards_gather_reduce_and_step(tmp_path):
    out = str(tmp_path / "r.pt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["n_units"] >= 2
    assert r["gather_ok"] and r["grad_ok"]
    assert r["step_err"] < 1e-6
    assert r["ckpt_ok"]


def test_fsdp_needs_fused_layers():
    from sigma0_b200.models import preset_args
    from sigma0_b200.models.registry import build_model
    from sigma0_b200.parallel.fsdp import FSDP
    model = build_model(preset_args("smoke", impl="torch", d_model=64, mamba3_d_state=16, mamba3_headdim=16))
    with pytest.raises(ValueError):
        FSDP(model, 2, 0)
