"""tcgen05 GEMM vs cuBLAS on the projection shapes of a training step.

    python -m sigma0_b200.eval.gemm_bench --tokens 88000 --d_model 1024 --d_proj 4384 --d_inner 2048

For every product of one Mamba3 layer (in_proj, out_proj and the GLU gate; forward, input
gradient, weight gradient) it times this package's GEMM and ``torch.matmul`` (cuBLAS) with
CUDA events (warm-up first; the token-sized operands are larger than L2) and prints one
JSON line per shape with both rates in TFLOP/s and the numeric agreement.
"""
from __future__ import annotations

import argparse
import json


def _time(fn, warmup: int, iters: int) -> float:
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None):
    import torch
    from ..ops import gemm
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--tokens", type=int, default=88000)
    ap.add_argument("--d_model", type=int, default=1024)
    ap.add_argument("--d_proj", type=int, default=4384)
    ap.add_argument("--d_inner", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--only", default=None, help="comma-separated product names")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    T, H, P, I = a.tokens, a.d_model, a.d_proj, a.d_inner
    g = torch.Generator(device=dev).manual_seed(0)
    r = lambda *s: (torch.randn(*s, device=dev, generator=g) * 0.05).bfloat16()
    shapes = [("in_proj", H, P), ("out_proj", I, H), ("glu_gate", H, H)]
    only = set(a.only.split(",")) if a.only else None
    for name, k, n in shapes:
        x, w, dy = r(T, k), r(k, n), r(T, n)
        acc = torch.zeros(k, n, device=dev)
        cases = [
            (f"{name}.fwd", 2.0 * T * k * n, lambda: gemm.mm(x, w), lambda: x @ w, lambda: x.float() @ w.float()),
            (f"{name}.dx", 2.0 * T * k * n, lambda: gemm.mm_nt(dy, w), lambda: dy @ w.t(),
             lambda: dy.float() @ w.float().t()),
            (f"{name}.dw", 2.0 * T * k * n, lambda: gemm.mm_tn_acc(x, dy, acc), lambda: x.t() @ dy,
             lambda: x.float().t() @ dy.float()),
        ]
        for label, flops, ours, lib, ref in cases:
            if only and label not in only:
                continue
            if label.endswith(".dw"):
                acc.zero_()
                ours()
                got = acc.clone()
            else:
                got = ours()
            want = ref()
            rel = float((got.float() - want).norm() / want.norm())
            t_ours = _time(ours, a.warmup, a.iters)
            t_lib = _time(lib, a.warmup, a.iters)
            print(json.dumps({"product": label, "M": T if not label.endswith(".dw") else k,
                              "N": n if not label.endswith(".dx") else k, "K": k if not label.endswith(".dw") else T,
                              "ours_ms": round(t_ours, 4), "cublas_ms": round(t_lib, 4),
                              "ours_tflops": round(flops / t_ours / 1e9, 1), "cublas_tflops": round(flops / t_lib / 1e9, 1),
                              "ratio": round(t_lib / t_ours, 3), "rel_err": rel, "status": gemm.status(x)}), flush=True)


if __name__ == "__main__":
    main()
