"""Data-parallel gradient sync fused with the AdamW update over NVLink peer memory.

``FusedDPSync`` owns the symmetric (peer-mapped) buffers that the cooperative
kernel ``dp_fused_adam`` (``csrc/dp_fused.cu``) reads and writes: every rank's
flat gradient, flat fp32 parameters and bf16 shadow (allocated through
``torch.distributed._symmetric_memory`` and re-homed into the optimizer), plus
a flag block and sum-of-squares slots for the in-kernel cross-rank barriers.
One launch per step replaces NCCL reduce-scatter + norm all-reduce + Adam +
NCCL all-gather; the per-rank Adam moments cover only the rank's shard
(ZeRO-1/2 memory), exactly as in the NCCL sharded path of ``Trainer``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def symmetric_alloc(group=None):
    """An allocator ``(numel, dtype) -> zeroed tensor`` in symmetric memory."""
    import torch.distributed._symmetric_memory as symm

    def alloc(numel, dtype, device):
        t = symm.empty(numel, dtype=dtype, device=device)
        t.zero_()
        return t
    return alloc


class FusedDPSync:
    SPIN_LIMIT = 30_000_000   # polls of ~64 ns: a peer missing for ~2 s aborts the step

    def __init__(self, opt, group=None):
        import torch.distributed._symmetric_memory as symm
        self.opt = opt
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("the fused path handles at most 8 ranks (one NVLink domain)")
        dev = opt.device
        self.flags = symm.empty(3 * 8, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.sums = symm.empty(8, dtype=torch.float32, device=dev)
        self.sums.zero_()
        torch.cuda.synchronize(dev)
        hs = {}
        for name, t in (("G", opt.grad), ("P", opt.flat), ("S", opt.shadow), ("F", self.flags), ("Q", self.sums)):
            hs[name] = symm.rendezvous(t, self.group)
        base = lambda h, t: [int(p) + (t.data_ptr() - int(h.buffer_ptrs[h.rank])) for p in h.buffer_ptrs]
        self.G = base(hs["G"], opt.grad)
        self.P = base(hs["P"], opt.flat)
        self.S = base(hs["S"], opt.shadow)
        self.F = base(hs["F"], self.flags)
        self.Q = base(hs["Q"], self.sums)
        self._handles = hs
        self.scratch = torch.zeros(2, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        # every step copies the status word to pinned host memory behind the kernel; the next
        # step (or ``poll``) reads that copy, so a timed-out peer raises without a per-step
        # device synchronisation
        self._host_status = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._status_ev = torch.cuda.Event()
        self._pending = False
        self.seq = 0
        dist.barrier(group=self.group)

    def step(self, lr_scale: float) -> None:
        from ..ops._ext import ext
        self._check_previous()
        o = self.opt
        o.step_count += 1
        t = o.step_count
        self.seq += 1
        ext().dp_fused_adam(self.G, self.P, self.S, self.F, self.Q, o.m, o.v, self.scratch, self.status,
                            o.lo, o.hi, o.n_ssm, self.rank, self.seq, self.SPIN_LIMIT,
                            o.base_lr["ssm"] * lr_scale, o.base_lr["regular"] * lr_scale, o.wd, o.b1, o.b2, o.eps,
                            1 - o.b1 ** t, 1 - o.b2 ** t, o.max_grad_norm)
        self._host_status.copy_(self.status, non_blocking=True)
        self._status_ev.record()
        self._pending = True

    def _raise_if(self, s: int) -> None:
        if s:
            raise RuntimeError(f"fused data-parallel step: a peer did not arrive (phase {s - 100}); "
                               f"a rank has failed or left")

    def _check_previous(self) -> None:
        """Raise if the previous step's kernel reported a timed-out wait (waits for that
        step's status copy, which lags the host by at most one step)."""
        if self._pending:
            self._status_ev.synchronize()
            self._pending = False
            self._raise_if(int(self._host_status[0]))

    def poll(self) -> None:
        """Raise now if the last finished step reported a timed-out wait (non-blocking when
        the step is still running; the next ``step`` checks it then)."""
        if self._pending and self._status_ev.query():
            self._pending = False
            self._raise_if(int(self._host_status[0]))

    def check(self) -> None:
        """Raise if any in-kernel cross-rank wait timed out (reads one word; syncs the stream)."""
        self._pending = False
        self._raise_if(int(self.status.item()))
