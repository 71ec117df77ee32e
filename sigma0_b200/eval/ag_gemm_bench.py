"""FSDP's first projection: all-gather of the sharded kernel + GEMM, NCCL then GEMM against
the fused kernel that gathers the row blocks itself (``csrc/gemm_tc.cu`` ``ag_copy``).

    torchrun --nproc-per-node 2 -m sigma0_b200.eval.ag_gemm_bench --tokens 88000

Times both on the device with CUDA events (max over ranks) and reports the fused kernel
against its roofline: the slower of the GEMM at the measured peak and the bytes that must
cross NVLink (the (world - 1) / world of the kernel this GPU lacks) at 770 GB/s.
"""
from __future__ import annotations

import argparse
import json
import os


def main(argv=None):
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm
    from ..ops import gemm
    from ..ops._ext import ext
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=88000)
    ap.add_argument("--d_model", type=int, default=1024)
    ap.add_argument("--d_proj", type=int, default=4480)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    K, N, T = a.d_model, a.d_proj, a.tokens
    rows = K // world
    g = torch.Generator(device=dev).manual_seed(0)
    full_ref = (torch.randn(K, N, device=dev, generator=g) * 0.05).bfloat16()      # same on every rank
    shard = symm.empty(rows * N, dtype=torch.bfloat16, device=dev)
    shard.copy_(full_ref[rank * rows:(rank + 1) * rows].reshape(-1))
    ready = symm.empty(8, dtype=torch.int32, device=dev)
    ready.fill_(1)
    torch.cuda.synchronize()
    h, hr = symm.rendezvous(shard, dist.group.WORLD), symm.rendezvous(ready, dist.group.WORLD)
    src = [int(p) for p in h.buffer_ptrs]
    rdy = [int(p) + 4 * r for r, p in enumerate(hr.buffer_ptrs)]
    counters = torch.zeros(8, dtype=torch.int32, device=dev)
    x = (torch.randn(T, K, device=dev, generator=g) * 0.05).bfloat16()
    wfull = torch.empty(K, N, dtype=torch.bfloat16, device=dev)
    dist.barrier()

    def fused():
        return ext().gemm_ag(x, wfull, src, rdy, counters, rank, 1, 20_000_000)

    def nccl():
        dist.all_gather_into_tensor(wfull.view(-1), shard)
        return gemm.mm(x, wfull)

    y = fused()
    torch.cuda.synchronize()
    err = float((y.float() - x.float() @ full_ref.float()).norm() / (x.float() @ full_ref.float()).norm())
    gathered_ok = bool(torch.equal(wfull, full_ref))

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)
    t_fused, t_nccl = timed(fused), timed(nccl)
    flops = 2.0 * T * K * N
    nv_bytes = (world - 1) / world * K * N * 2
    from ..models.flops import measured_bf16_peak
    roof_ms = max(flops / measured_bf16_peak(sustained=False), nv_bytes / 770e9) * 1e3
    if rank == 0:
        print(json.dumps({"world": world, "tokens": T, "K": K, "N": N, "fused_ms": round(t_fused, 4),
                          "nccl_then_gemm_ms": round(t_nccl, 4), "speedup": round(t_nccl / t_fused, 3),
                          "roofline_ms": round(roof_ms, 4), "fused_frac_of_roofline": round(roof_ms / t_fused, 3),
                          "rel_err": err, "gathered_exact": gathered_ok, "status": gemm.status(x)}), flush=True)
    del h, hr
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
