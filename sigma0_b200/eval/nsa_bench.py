"""Time an NSA block with its branches on the flash kernels against the tensor-expression path.

    python -m sigma0_b200.eval.nsa_bench [--B 1 --L 16384 --H 1024 --nh 16 --bs 32 --sb 64 --top 16]

Forward and forward + backward of one ``NSABlock`` (bf16 compute, compression block
``--bs``, selection block ``--sb``, ``--top`` selected blocks, full-causal third branch)
with ``ops.attention.use_kernels(True / False)``, CUDA events after warm-up, plus the
relative difference of the outputs and the peak memory of each path.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--L", type=int, default=16384)
    ap.add_argument("--H", type=int, default=1024)
    ap.add_argument("--nh", type=int, default=16)
    ap.add_argument("--bs", type=int, default=32)
    ap.add_argument("--sb", type=int, default=64)
    ap.add_argument("--top", type=int, default=16)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args(argv)
    from ..models.nsa import NSABlock
    from ..ops.attention import use_kernels
    torch.manual_seed(0)
    m = NSABlock(a.H, n_heads=a.nh, block_size=a.bs, select_block=a.sb, block_counts=a.top,
                 dtype=torch.bfloat16).cuda()
    x = torch.randn(a.B, a.L, a.H, device="cuda", requires_grad=True)
    out = {"B": a.B, "L": a.L, "H": a.H, "nh": a.nh, "block": a.bs, "select_block": a.sb, "top": a.top}
    outs = {}
    for name, on in (("kernels", True), ("torch", False)):
        with use_kernels(on):
            with torch.no_grad():
                tf = _time(lambda: m(x), a.iters, a.warmup)
                outs[name] = m(x).float()

            def fb():
                x.grad = None
                m(x).sum().backward()
            torch.cuda.reset_peak_memory_stats()
            tfb = _time(fb, a.iters, a.warmup)
            out[name] = {"fwd_ms": tf, "fwd_bwd_ms": tfb, "peak_gb": torch.cuda.max_memory_allocated() / 1e9}
    r = outs["torch"] - x.detach()
    out["rel_diff"] = ((outs["kernels"] - outs["torch"]).norm() / r.norm()).item()
    out["speedup_fwd_bwd"] = out["torch"]["fwd_bwd_ms"] / out["kernels"]["fwd_bwd_ms"]
    print(json.dumps(out))


if __name__ == "__main__":
    main()
