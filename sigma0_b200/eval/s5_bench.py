"""Time an S5 layer with the scan kernels against the chunked einsum path.

    python -m sigma0_b200.eval.s5_bench [--B 8 --L 13000 --H 512 --state 512 --blocks 8]

Forward and forward + backward of one S5 layer (``make_s5_factory``), CUDA events after
warm-up, with ``S5.use_kernel`` on and off, plus the relative difference of the outputs.
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
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--L", type=int, default=13000)
    ap.add_argument("--H", type=int, default=512)
    ap.add_argument("--state", type=int, default=512)
    ap.add_argument("--blocks", type=int, default=8)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args(argv)
    from ..models.s5 import make_s5_factory
    torch.manual_seed(0)
    m = make_s5_factory(a.state, a.blocks)(a.H).cuda()
    u = torch.randn(a.B, a.L, a.H, device="cuda", requires_grad=True)
    out = {"B": a.B, "L": a.L, "H": a.H, "P": m.P}
    ys = {}
    for name, on in (("kernel", True), ("einsum", False)):
        m.use_kernel = on
        with torch.no_grad():
            tf = _time(lambda: m(u), a.iters, a.warmup)
            ys[name] = m(u)

        def fb():
            u.grad = None
            m.zero_grad(set_to_none=True)
            m(u).sum().backward()
        out[name] = {"fwd_ms": tf, "fwd_bwd_ms": _time(fb, a.iters, a.warmup)}
    out["rel_diff"] = ((ys["kernel"] - ys["einsum"]).norm() / ys["einsum"].norm()).item()
    out["speedup_fwd_bwd"] = out["einsum"]["fwd_bwd_ms"] / out["kernel"]["fwd_bwd_ms"]
    print(json.dumps(out))


if __name__ == "__main__":
    main()
