"""Time the sm_100a flash attention kernels against torch's attention.

    python -m sigma0_b200.eval.attn_bench [--B 2 --L 8192 --nh 16 --hd 64 --window 512]

For each mode (full causal; sliding window when ``--window`` > 0) it times forward and
forward + backward of ``ops.attention.flash_attention`` (the repo's kernels) and of the
torch path it replaces (scaled_dot_product_attention with is_causal -- torch picks its
fastest backend -- for causal; the blocked masked softmax for a window), with CUDA events
after warm-up, and reports TFLOP/s of the visible score entries (4 * hd FLOPs per entry
forward, 2.5x that for forward + backward).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F


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
    ap.add_argument("--B", type=int, default=2)
    ap.add_argument("--L", type=int, default=8192)
    ap.add_argument("--nh", type=int, default=16)
    ap.add_argument("--hd", type=int, default=64)
    ap.add_argument("--window", type=int, default=512)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    from ..ops import attention as A
    B, L, nh, hd = a.B, a.L, a.nh, a.hd
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, L, nh, hd, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
               for _ in range(3))
    do = torch.randn(B, L, nh, hd, device="cuda", generator=g).to(torch.bfloat16)
    modes = [("causal", None)] + ([("window", a.window)] if a.window > 0 else [])
    out = {"B": B, "L": L, "nh": nh, "hd": hd}
    for name, w in modes:
        if w is None:
            entries = B * nh * L * (L + 1) / 2

            def torch_fwd():
                return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                      is_causal=True).transpose(1, 2)
        else:
            entries = B * nh * sum(min(i + 1, w) for i in range(L))

            def torch_fwd():
                return A._blocked(q, k, v, hd ** -0.5, w, 0)

        def ours_fwd():
            return A.flash_attention(q, k, v, window=w, force_kernel=True)

        res = {}
        for impl, fwd in (("ours", ours_fwd), ("torch", torch_fwd)):
            with torch.no_grad():
                tf = _time(fwd, a.iters, a.warmup)

            def fb():
                q.grad = k.grad = v.grad = None
                fwd().backward(do)
            tfb = _time(fb, a.iters, a.warmup)
            res[impl] = {"fwd_ms": tf, "fwd_bwd_ms": tfb, "fwd_tflops": 4 * hd * entries / tf / 1e9,
                         "fwd_bwd_tflops": 10 * hd * entries / tfb / 1e9}
        with torch.no_grad():
            err = ((ours_fwd().float() - torch_fwd().float()).norm() / torch_fwd().float().norm()).item()
        res["rel_diff_fwd"] = err
        out[name if w is None else f"window{w}"] = res
    print(json.dumps(out))


if __name__ == "__main__":
    main()
