"""Time the chunked gated delta rule with the CUDA state scan against the host loop.

    python -m sigma0_b200.eval.gdn_bench [--B 1 --L 8192 --nh 8 --hd 128 --hvd 256 --kda]

Forward and forward + backward of ``models.gdn.gated_delta_chunked`` (chunk 64) with
``use_kernel=True`` (csrc/gdn_scan.cu for the cross-chunk scan) and ``False`` (one
batched step per chunk from the host), CUDA events after warm-up, plus the relative
difference of the outputs.
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
    ap.add_argument("--L", type=int, default=8192)
    ap.add_argument("--nh", type=int, default=8)
    ap.add_argument("--hd", type=int, default=128)
    ap.add_argument("--hvd", type=int, default=256)
    ap.add_argument("--kda", action="store_true")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args(argv)
    from ..models.gdn import gated_delta_chunked, l2_normalize
    g = torch.Generator(device="cuda").manual_seed(0)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    B, L, nh, hd, hvd = a.B, a.L, a.nh, a.hd, a.hvd
    q = (l2_normalize(r(B, L, nh, hd)) * hd ** -0.5).requires_grad_(True)
    k = l2_normalize(r(B, L, nh, hd)).requires_grad_(True)
    v = r(B, L, nh, hvd).requires_grad_(True)
    beta = torch.sigmoid(r(B, L, nh)).requires_grad_(True)
    alog = torch.nn.functional.logsigmoid(r(B, L, nh, hd if a.kda else 1) + 3.0).requires_grad_(True)
    do = r(B, L, nh, hvd)
    out = {"B": B, "L": L, "nh": nh, "hd": hd, "hvd": hvd, "kda": a.kda}
    res = {}
    for name, uk in (("kernel_scan", True), ("host_loop", False)):
        def fwd():
            return gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=uk)[0]
        with torch.no_grad():
            tf = _time(fwd, a.iters, a.warmup)

        def fb():
            for t in (q, k, v, beta, alog):
                t.grad = None
            fwd().backward(do)
        res[name] = {"fwd_ms": tf, "fwd_bwd_ms": _time(fb, a.iters, a.warmup)}
    with torch.no_grad():
        o1 = gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=True)[0]
        o2 = gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=False)[0]
    out.update(res, rel_diff=((o1 - o2).norm() / o2.norm()).item(),
               speedup_fwd_bwd=res["host_loop"]["fwd_bwd_ms"] / res["kernel_scan"]["fwd_bwd_ms"])
    print(json.dumps(out))


if __name__ == "__main__":
    main()
