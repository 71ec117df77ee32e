"""Time the fused tensor-parallel projection + all-reduce against GEMM + NCCL all-reduce.

Run one process per GPU (``torchrun --nproc-per-node W -m sigma0_b200.parallel.tp_bench``);
without torchrun it runs the single-rank kernel (no peers) for profiling the GEMM part.
Shape: ``--tokens`` rows, the rank's ``--k_total / W`` columns of a row-parallel
projection to ``--n_out`` outputs (the Mamba3 out_proj of d_model 1024: K = 2048 split
over W ranks, N = 1024).  Each variant is timed with CUDA events after warm-up, the max
over ranks is reported, plus the roofline of the fused kernel: the slower of its FLOPs at
the measured GEMM peak and the bytes each rank must push over NVLink (fp32 partial tiles
to their owners, bf16 owned rows to every peer) at the measured 770 GB/s per direction.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--k_total", type=int, default=2048)
    ap.add_argument("--n_out", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--gemm_tflops", type=float, default=1639.5)
    ap.add_argument("--link_gbs", type=float, default=770.0)
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    multi = "WORLD_SIZE" in os.environ
    if multi:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    W, r = (dist.get_world_size(), dist.get_rank()) if multi else (1, 0)
    sync = (lambda: dist.barrier()) if multi else (lambda: None)
    from .tp_fused import FusedRowParallel
    K = a.k_total // W
    g = torch.Generator(device="cuda").manual_seed(r)
    y = torch.randn(a.tokens, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(K, a.n_out, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    wt = w.t().contiguous()
    h = FusedRowParallel(a.tokens, a.n_out)

    def fused():
        return h(y, wt, copy=False)

    def nccl():
        o = y @ w
        if multi:
            dist.all_reduce(o)
        return o

    res = {}
    for name, fn in (("fused", fused), ("gemm_nccl_bf16" if multi else "gemm_cublas", nccl)):
        for _ in range(a.warmup):
            fn()
        sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.iters], device="cuda")
        if multi:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name + "_ms"] = float(t)
    h.check()
    stamps = torch.zeros(4 + torch.cuda.get_device_properties(0).multi_processor_count, dtype=torch.int64,
                         device="cuda")
    sync()
    h(y, wt, copy=False, stamps=stamps)
    torch.cuda.synchronize()
    res["fused_phases"] = FusedRowParallel.phase_times(stamps)
    ref = y.float() @ w.float()
    if multi:
        dist.all_reduce(ref)
    err = float((h(y, wt).float() - ref).norm() / ref.norm())
    flops = 2.0 * a.tokens * K * a.n_out
    link = (W - 1) / W * a.tokens * a.n_out * 2 + (W - 1) * (a.tokens / W) * a.n_out * 2   # bf16 both ways
    roof_ms = max(flops / (a.gemm_tflops * 1e12), link / (a.link_gbs * 1e9)) * 1e3
    res.update(world=W, tokens=a.tokens, k_per_rank=K, n_out=a.n_out, rel_err_vs_fp32=err,
               roofline_ms=roof_ms, fused_fraction_of_roofline=roof_ms / res["fused_ms"],
               nvlink_bytes_per_rank=link)
    if r == 0:
        print(json.dumps(res))
    if multi:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
