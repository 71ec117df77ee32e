"""Mamba3 SSD kernels versus the fp32 torch oracle: parity, then speed.

The counterpart of the reference's SSD kernel bench
(``run/base_model/bench/ssd_kernel_bench.py:1-311``: fused Pallas SSD against its
XLA reference).  For one geometry it

1. checks parity on a short sequence: the CUDA forward output and every gradient
   of the CUDA backward (the projection columns z, x, B, C, dt, A, trapezoid,
   angles and the six SSD parameters) against autograd through the chunked fp32
   oracle (``ops/reference/mamba3_ref.py``), as relative L2 errors;
2. times, with CUDA events after warm-up, the CUDA forward alone and
   forward + backward at the full length, and the oracle's forward and
   forward + backward for comparison (skipped with ``--no_oracle_speed``).

The kernels take the model's projection rows (``[B*L, ldp]`` bf16: z | x | B | C |
dt | A | trap | angle columns), so inputs are drawn in that layout; B, C and the
angle rates are shared by all heads as in the model.  One JSON record per
configuration goes to stdout::

    python -m sigma0_b200.eval.ssd_bench --L 13000 --nh 32
"""
from __future__ import annotations

import argparse
import json
import statistics
from typing import Callable, Dict, List

import torch


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


def _layer(nh: int, seed: int):
    from ..models.mamba3 import Mamba3
    torch.manual_seed(seed)
    H = nh * 64 // 2                         # expand 2, headdim 64
    m = Mamba3(H, impl="cuda").cuda()
    with torch.no_grad():
        m.B_bias.normal_(0, 0.5)
        m.C_bias.normal_(0, 0.5)
        m.D.normal_(1, 0.2)
        m.B_norm.scale.normal_(1, 0.1)
        m.C_norm.scale.normal_(1, 0.1)
    return m


def _proj(m, B: int, L: int, seed: int) -> torch.Tensor:
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    g = torch.Generator(device="cuda").manual_seed(seed)
    p = (torch.randn(B * L, ldp, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    p[:, d.d_in_proj:] = 0
    return p


def _oracle_y(m, proj32: torch.Tensor, B: int, L: int) -> torch.Tensor:
    from ..ops.reference import mamba3_ref as ref
    z, x, Bn, Cn, ADT, DT, trap, ang = m._prep(proj32.view(B, L, -1))
    nh = m.dims.n_heads
    y = ref.mamba3_ssd_chunked(Cn[:, :, None].expand(-1, -1, nh, -1), Bn[:, :, None].expand(-1, -1, nh, -1), x,
                               ADT.transpose(1, 2), DT.transpose(1, 2), trap.transpose(1, 2), ang, m.C_bias,
                               m.B_bias, m.D, z, chunk_size=m.dims.chunk_size)
    return y.reshape(B * L, -1)


def _cuda_fwd(m, proj, B, L):
    from ..ops._ext import ext
    d = m.dims
    return ext().m3_fwd(proj, B, L, d.n_heads, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias,
                        m.D, m.A_floor, m.B_norm.eps)[0]


def _cuda_bwd(m, proj, dy, B, L):
    from ..ops._ext import ext
    d = m.dims
    return ext().m3_bwd(proj, dy, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D, B, L,
                        d.n_heads, m.A_floor, m.B_norm.eps)


def parity(nh: int, L: int, B: int = 1, seed: int = 0) -> Dict[str, float]:
    """Relative L2 errors of the CUDA forward and backward against the fp32 oracle."""
    m = _layer(nh, seed)
    d = m.dims
    proj = _proj(m, B, L, seed + 1)
    dy = (torch.randn(B * L, d.d_inner, device="cuda") * 0.5).to(torch.bfloat16)
    y = _cuda_fwd(m, proj, B, L)
    dproj, dwB, dwC, ddtb, dD, dCb, dBb = _cuda_bwd(m, proj, dy, B, L)
    p32 = proj[:, :d.d_in_proj].float().clone().requires_grad_(True)
    params = [m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.D, m.C_bias, m.B_bias]
    for p in params:
        p.grad = None
    yr = _oracle_y(m, p32, B, L)
    (yr * dy.float()).sum().backward()
    out = {"y": _rel(y.view(B * L, -1), yr)}
    sizes = [("dz", d.d_inner), ("dx", d.d_inner), ("dB", d.d_state), ("dC", d.d_state), ("d_dt", d.n_heads),
             ("d_A", d.n_heads), ("d_trap", d.n_heads), ("d_angle", d.R)]
    off = 0
    for name, s in sizes:
        out[name] = _rel(dproj[:, off:off + s], p32.grad[:, off:off + s])
        off += s
    for got, p, name in [(dwB, m.B_norm.scale, "d_B_norm"), (dwC, m.C_norm.scale, "d_C_norm"),
                         (ddtb, m.dt_bias, "d_dt_bias"), (dD, m.D, "d_D"), (dCb, m.C_bias, "d_C_bias"),
                         (dBb, m.B_bias, "d_B_bias")]:
        out[name] = _rel(got, p.grad)
    return out


def _time_ms(fn: Callable[[], object], warmup: int, iters: int) -> List[float]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b))
    return out


def speed(nh: int, L: int, B: int = 1, warmup: int = 3, iters: int = 10, oracle: bool = True,
          seed: int = 0) -> Dict[str, float]:
    """Median milliseconds of the CUDA forward and forward+backward (and the oracle's)."""
    m = _layer(nh, seed)
    d = m.dims
    proj = _proj(m, B, L, seed + 1)
    dy = (torch.randn(B * L, d.d_inner, device="cuda") * 0.5).to(torch.bfloat16)
    res = {}
    with torch.no_grad():
        res["cuda_fwd_ms"] = statistics.median(_time_ms(lambda: _cuda_fwd(m, proj, B, L), warmup, iters))
    res["cuda_fwd_bwd_ms"] = statistics.median(
        _time_ms(lambda: (_cuda_fwd(m, proj, B, L), _cuda_bwd(m, proj, dy, B, L)), warmup, iters))
    tokens = B * L
    res["cuda_fwd_bwd_tokens_per_s"] = tokens / (res["cuda_fwd_bwd_ms"] * 1e-3)
    if oracle:
        p32 = proj[:, :d.d_in_proj].float()
        with torch.no_grad():
            res["oracle_fwd_ms"] = statistics.median(_time_ms(lambda: _oracle_y(m, p32, B, L), 1, 3))

        def fb():
            p = p32.clone().requires_grad_(True)
            (_oracle_y(m, p, B, L) * dy.float()).sum().backward()
        res["oracle_fwd_bwd_ms"] = statistics.median(_time_ms(fb, 1, 3))
        res["speedup_fwd_bwd"] = res["oracle_fwd_bwd_ms"] / res["cuda_fwd_bwd_ms"]
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--L", type=int, nargs="+", default=[13000])
    ap.add_argument("--nh", type=int, default=32)
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--parity_L", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no_oracle_speed", action="store_true")
    ap.add_argument("--skip_parity", action="store_true", help="timings only (e.g. under a profiler)")
    ap.add_argument("--impl", choices=["auto", "walker", "chunked"], default="auto",
                    help="walker: the tcgen05 chunk walkers; chunked: the chunk-parallel mma.sync kernels; "
                         "auto: the walkers when (sequences x heads) >= SMs")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("the SSD kernel bench needs a CUDA device")
    from ..ops._ext import ext
    ext().m3_use_tc(None if a.impl == "auto" else a.impl == "walker")
    par = None if a.skip_parity else parity(a.nh, a.parity_L)
    for L in a.L:
        rec = {"impl": a.impl, "nh": a.nh, "N": 128, "P": 64, "CS": 64, "B": a.B, "L": L, "parity_L": a.parity_L,
               "parity_rel_l2": par}
        rec.update(speed(a.nh, L, a.B, a.warmup, a.iters, oracle=not a.no_oracle_speed))
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
