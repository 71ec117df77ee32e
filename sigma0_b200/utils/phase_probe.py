"""Per-phase cycle counts of the Mamba3 chunk-backward kernel.

Needs the extension built with the probe counters compiled in
(``S0_PHASE_PROBE=1 python setup.py build_ext --inplace``; the default build has
none and this tool then says so).  Runs the mixer forward and backward of one
350m-sized Mamba3 layer (d_model 1024, 32 heads) on ``--B`` x ``--L`` tokens and
prints the mean cycles per block of every phase, as measured by thread 0 of each
block with ``clock64()`` (phase boundaries are block barriers, so thread 0's view
is the block's).

    python -m sigma0_b200.utils.phase_probe --B 2 --L 11000
"""
from __future__ import annotations

import argparse

PHASES = {0: "load (scalar group + tile wait start)", 8: "row scalars", 9: "angles + tile wait",
          10: "dY0 + Q/K build", 1: "prologue tail", 2: "A: QK^T, Q S^T, dY0 V^T -> P, dS",
          3: "B: P V -> y0 -> dz", 11: "C+D: GEMMs", 12: "C+D: epilogue", 7: "C+D: reductions",
          4: "barrier after C+D", 5: "E: dV + S_out dot", 6: "F: stores and scans"}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--B", type=int, default=2)
    ap.add_argument("--L", type=int, default=11000)
    ap.add_argument("--iters", type=int, default=4)
    a = ap.parse_args(argv)
    import torch
    from ..models.mamba3 import Mamba3
    from ..ops._ext import ext
    from ..ops.mamba3_layer import mamba3_mixer
    if ext().m3_phase_probe().numel() == 0:
        raise SystemExit("this build has no phase counters: rebuild with S0_PHASE_PROBE=1")
    torch.manual_seed(0)
    m = Mamba3(1024, impl="cuda").cuda()
    u = (torch.randn(a.B, a.L, 1024, device="cuda") * 0.5).requires_grad_(True)
    for _ in range(a.iters):
        mamba3_mixer(u, m).float().square().mean().backward()
        torch.cuda.synchronize()
        v = ext().m3_phase_probe()        # counters of the last iteration only
    blocks = a.B * ((a.L + 63) // 64) * m.dims.n_heads
    total = sum(int(v[k]) for k in PHASES) / blocks
    print(f"blocks {blocks}, mean cycles per block {total:.0f}")
    for k, name in PHASES.items():
        c = int(v[k]) / blocks
        print(f"{name:40s} {c:8.0f} cycles  {100 * c / total:5.1f}%")


if __name__ == "__main__":
    main()
