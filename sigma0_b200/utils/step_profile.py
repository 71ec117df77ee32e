"""Kernel-time breakdown of one training step (torch profiler, CUDA activity only).

Builds the preset's model and trainer on ``cuda:0`` with synthetic sequences of the
preset's shape, runs ``--warmup`` steps, profiles one step and prints every kernel's
share of the step's device time, launch count and mean duration.  The table explains
where a step's time goes; it is not a benchmark (the profiler adds overhead; time
steps with ``bench.py``).

    python -m sigma0_b200.utils.step_profile --preset 350m --top 30

``TraceWindow`` is the training loop's trace hook: the reference starts a JAX profiler
trace at step 2 and stops it at step 20 under ``--enable_profiler``
(``training/train_helpers.py:1033-1034,1229-1231``); here a ``torch.profiler`` session
covers the same optimizer-step window (CPU and CUDA activity) and writes one Chrome trace
per rank, and NVTX ranges mark every step for an external timeline tool.
"""
from __future__ import annotations

import argparse
import collections
from typing import Dict, List, Optional, Tuple


class TraceWindow:
    """Profile optimizer steps ``[start, stop)``; ``trace_rank{r}.json`` goes to ``out_dir``."""

    def __init__(self, start: int, stop: int, out_dir: str, rank: int = 0, nvtx: bool = False):
        if stop <= start:
            raise ValueError(f"empty profiler window [{start}, {stop})")
        self.start, self.stop, self.out_dir, self.rank, self.nvtx = int(start), int(stop), out_dir, rank, nvtx
        self.prof = None
        self.path: Optional[str] = None

    def before(self, step: int) -> None:
        """Call before optimizer step ``step`` (0-based) is issued."""
        import torch
        if step == self.start and self.prof is None:
            from torch.profiler import ProfilerActivity, profile
            acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
            self.prof = profile(activities=acts, record_shapes=False)
            self.prof.__enter__()
        if self.nvtx and torch.cuda.is_available():
            torch.cuda.nvtx.range_push(f"step {step}")

    def after(self, step: int) -> None:
        """Call after optimizer step ``step`` (0-based) has been issued."""
        import torch
        if self.nvtx and torch.cuda.is_available():
            torch.cuda.nvtx.range_pop()
        if self.prof is not None and step + 1 >= self.stop:
            self.close()

    def close(self) -> None:
        import os
        import torch
        if self.prof is None:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        os.makedirs(self.out_dir, exist_ok=True)
        self.path = os.path.join(self.out_dir, f"trace_rank{self.rank}.json")
        self.prof.export_chrome_trace(self.path)
        self.prof = None


def profile_step(preset: str = "350m", micro_bsz: int = 0, n_messages: int = 0,
                 warmup: int = 3) -> Tuple[float, List[Tuple[str, int, float]]]:
    """(total kernel ms, [(kernel, launches, total us)] sorted by time)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from ..data import LobWindowDataset, collate, make_sequences
    from ..models import preset_args
    from ..train.trainer import Trainer

    dev = torch.device("cuda", 0)
    args = preset_args(preset, impl="cuda")
    if micro_bsz:
        args.micro_bsz = micro_bsz
    if n_messages:
        args.n_messages = n_messages
    tr = Trainer(args, device=dev, world=1, rank=0, total_steps=10_000, seed=0)
    days = make_sequences(args.micro_bsz, args.n_messages + 1, seed=1000)
    ds = LobWindowDataset.from_days(days, args.n_messages, token_mode=args.token_mode)
    batch = tuple(t.to(dev) for t in collate([ds[i] for i in range(args.micro_bsz)]))
    for _ in range(warmup):
        tr.step_device(*batch)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        tr.step_device(*batch)
        torch.cuda.synchronize()
    agg: Dict[str, List[float]] = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if e.device_type.name == "CUDA":
            agg[e.name][0] += 1
            agg[e.name][1] += e.device_time_total
    rows = sorted(((k, int(v[0]), float(v[1])) for k, v in agg.items()), key=lambda r: -r[2])
    return sum(r[2] for r in rows) / 1000.0, rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--preset", default="350m")
    ap.add_argument("--micro_bsz", type=int, default=0)
    ap.add_argument("--n_messages", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--top", type=int, default=30)
    a = ap.parse_args(argv)
    total, rows = profile_step(a.preset, a.micro_bsz, a.n_messages, a.warmup)
    print(f"kernel time of one step: {total:.1f} ms")
    print(f"{'share':>6} {'launches':>8} {'mean us':>9}  kernel")
    for name, n, us in rows[:a.top]:
        print(f"{100 * us / (total * 1000):5.1f}% {n:8d} {us / n:9.1f}  {name[:110]}")


if __name__ == "__main__":
    main()
