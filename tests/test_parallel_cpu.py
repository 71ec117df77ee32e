"""Tensor and context parallelism of the Mamba3 mixer on CPU ranks (gloo, world 2)
against the single-process model: outputs and gradients."""
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


def close(a, b, tol=2e-5):
    return ((a - b).norm() / (b.norm() + 1e-12)).item() < tol


def _mixer():
    from sigma0_b200.models.mamba3 import Mamba3
    torch.manual_seed(0)
    m = Mamba3(64, d_state=16, headdim=16, chunk_size=16)
    with torch.no_grad():
        m.B_bias.normal_(0, 0.5)
        m.C_bias.normal_(0, 0.5)
        m.in_proj.kernel.mul_(3.0)
    return m


def _data(L=80):
    g = torch.Generator().manual_seed(1)
    return torch.randn(2, L, 64, generator=g, dtype=torch.float32), torch.randn(2, L, 64, generator=g)


def _reference(L=80):
    m = _mixer()
    u, gout = _data(L)
    u.requires_grad_(True)
    y = m(u)
    (y * gout).sum().backward()
    return m, u, y.detach()


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        torch.set_num_threads(1)
        u, gout = _data()
        if mode == "tp":
            from sigma0_b200.parallel.tp import Mamba3TP
            m = Mamba3TP(_mixer())
            u = u.clone().requires_grad_(True)
            y = m(u)
            (y * gout).sum().backward()
            res = {"y": y.detach(), "du": u.grad, "gin": m.full_in_proj_grad(), "gout_proj": m.out_proj_kernel.grad,
                   "h0": m.h0, "nhl": m.nhl, "gBn": m.B_norm_scale.grad, "gD": m.D.grad}
        else:
            from sigma0_b200.parallel.cp import Mamba3CP, split_sequence
            m = Mamba3CP(_mixer())
            us = split_sequence(u).clone().requires_grad_(True)
            y = m(us)
            (y * split_sequence(gout)).sum().backward()
            grads = {n: p.grad.clone() for n, p in m.inner.named_parameters()}
            for g in grads.values():
                dist.all_reduce(g)
            res = {"y": y.detach(), "du": us.grad, "grads": grads}
        torch.save(res, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


def _run(mode, tmp_path):
    out = str(tmp_path / "r")
    mp.spawn(_worker, args=(2, _port(), mode, out), nprocs=2, join=True)
    return [torch.load(f"{out}.{r}") for r in range(2)]


def test_tensor_parallel_mixer_matches_full(tmp_path):
    m, u, y = _reference()
    res = _run("tp", tmp_path)
    for r in res:
        assert close(r["y"], y)
        assert close(r["du"], u.grad)
        assert close(r["gBn"], m.B_norm.scale.grad)   # replicated weights: full grad
    P = m.dims.headdim
    full_in = m.in_proj.kernel.grad
    gsum = res[0]["gin"].clone()
    gsum[:, :] = 0
    for r in res:
        gsum += r["gin"]
    # head columns come from one rank each, shared columns are identical on both ranks
    d = m.dims
    shared = torch.cat([torch.arange(2 * d.d_inner, 2 * d.d_inner + 2 * d.d_state),
                        torch.arange(d.d_in_proj - d.R, d.d_in_proj)])
    gsum[:, shared] /= 2
    assert close(gsum, full_in)
    for r in res:
        h0, n = r["h0"], r["nhl"]
        assert close(r["gout_proj"], m.out_proj.kernel.grad[h0 * P:(h0 + n) * P])
        assert close(r["gD"], m.D.grad[h0:h0 + n])


def test_context_parallel_mixer_matches_full(tmp_path):
    m, u, y = _reference()
    res = _run("cp", tmp_path)
    L = y.shape[1] // 2
    for r, out in enumerate(res):
        assert close(out["y"], y[:, r * L:(r + 1) * L]), r
        assert close(out["du"], u.grad[:, r * L:(r + 1) * L]), r
    for n, p in m.named_parameters():
        assert close(res[0]["grads"][n], p.grad), n
