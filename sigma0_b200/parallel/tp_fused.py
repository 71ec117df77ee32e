"""Row-parallel projection + all-reduce as one kernel over NVLink peer memory.

``FusedRowParallel`` owns the symmetric (peer-mapped) buffers of the cooperative
kernel ``tp_gemm_allreduce`` (``csrc/tp_fused.cu``): every rank's receive slots
(one bf16 partial per source rank for the rows it owns), bf16 output buffer and
flag words.  A call computes ``out = sum_r y_r @ w_r`` over the tensor-parallel
group -- each rank's tcgen05 tiles are stored into the owner rank's slot while
later tiles are still being multiplied, the owners sum their slots in fp32 and
all-gather bf16 rows with peer stores -- replacing ``GEMM -> NCCL all-reduce``
(``reduce_from_tp``); the bytes crossing NVLink equal those of a bf16 ring.

``fused_row_parallel(y, w, helper)`` is the autograd form used by ``Mamba3TP``:
the all-reduce's backward is the identity, so dy = dout w^T and dw = y^T dout are
local.  With one rank the same kernel runs on plain buffers (no peers).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

BM, BN, BK = 128, 128, 64


def _ceil(a: int, b: int) -> int:
    return (a + b - 1) // b * b


class FusedRowParallel:
    SPIN_LIMIT = 30_000_000      # polls of ~64 ns: a peer missing for ~2 s aborts the call

    def __init__(self, max_rows: int, n_out: int, group=None, device=None):
        if n_out % BN:
            raise ValueError(f"output width {n_out} must be a multiple of {BN}")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("the fused path handles at most 8 ranks (one NVLink domain)")
        self.device = torch.device(device or "cuda")
        self.M, self.N = _ceil(max_rows, BM), n_out
        self.rows_own = _ceil(self.M // BM, self.world) // self.world * BM      # row tiles dealt round robin
        n_recv = self.world * self.rows_own * self.N
        if self.world > 1:
            import torch.distributed._symmetric_memory as symm
            self.recv = symm.empty(n_recv, dtype=torch.bfloat16, device=self.device)
            self.out = symm.empty(self.M * self.N, dtype=torch.bfloat16, device=self.device)
            self.flags = symm.empty(2 * 8, dtype=torch.int32, device=self.device)
            for t in (self.recv, self.out, self.flags):
                t.zero_()
            torch.cuda.synchronize(self.device)
            g = group or dist.group.WORLD
            bufs = (self.recv, self.out, self.flags)
            hs = [symm.rendezvous(t, g) for t in bufs]
            ptrs = lambda h, t: [int(p) + (t.data_ptr() - int(h.buffer_ptrs[h.rank])) for p in h.buffer_ptrs]
            self.recv_p, self.out_p, self.flag_p = (ptrs(h, t) for h, t in zip(hs, bufs))
            self._handles = hs
            dist.barrier(group=group)
        else:
            self.recv = torch.zeros(n_recv, dtype=torch.bfloat16, device=self.device)
            self.out = torch.zeros(self.M * self.N, dtype=torch.bfloat16, device=self.device)
            self.flags = torch.zeros(2 * 8, dtype=torch.int32, device=self.device)
            self.recv_p, self.out_p, self.flag_p = ([self.recv.data_ptr()], [self.out.data_ptr()],
                                                    [self.flags.data_ptr()])
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.abort = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.seq = 0

    def __call__(self, y: torch.Tensor, w_t: torch.Tensor, copy: bool = True,
                 stamps: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [T, K] bf16 (this rank's columns), w_t [N, K] bf16 (this rank's rows of the
        projection, transposed) -> sum over ranks of y_r w_r, [T, N] bf16 (``copy=False``:
        a view of the output buffer, overwritten by the next call).  ``stamps`` (int64 CUDA,
        4 + SM count entries) receives %globaltimer stamps of the phases (see ``phase_times``)."""
        from ..ops._ext import ext
        T, K = y.shape
        if T > self.M or w_t.shape[0] != self.N or w_t.shape[1] != K or K % BK:
            raise ValueError(f"shape mismatch: y {tuple(y.shape)}, w_t {tuple(w_t.shape)}, buffers {self.M}x{self.N}")
        Mp = _ceil(T, BM)
        yp = y if (Mp == T and y.is_contiguous()) else torch.nn.functional.pad(y, (0, 0, 0, Mp - T)).contiguous()
        yp, w_t = yp.to(torch.bfloat16), w_t.to(torch.bfloat16).contiguous()
        # the operand tensor maps need 16-byte aligned bases
        yp = yp if yp.data_ptr() % 16 == 0 else yp.clone()
        w_t = w_t if w_t.data_ptr() % 16 == 0 else w_t.clone()
        self.seq += 1
        self.abort.zero_()
        rc = ext().tp_gemm_allreduce(yp, w_t, self.recv_p,
                                     self.rows_own, self.out_p, self.flag_p, self.rank, self.seq, self.SPIN_LIMIT,
                                     self.status, self.abort, stamps)
        if rc != 0:
            raise RuntimeError(f"tp_gemm_allreduce launch failed ({rc})")
        out = self.out[:T * self.N].view(T, self.N)
        return out.clone() if copy else out

    @staticmethod
    def phase_times(stamps: torch.Tensor) -> dict:
        """Microseconds per phase from a call's stamps: the slowest CTA's GEMM + reduce-scatter
        work, the spread of the CTAs' finish times, the wait at the cross-rank barrier, the
        owner sum + all-gather, and the closing barrier."""
        s = stamps.cpu().tolist()
        ctas = [v for v in s[4:] if v > 0]
        return {"gemm_scatter_us": (max(ctas) - s[0]) / 1e3, "cta_spread_us": (max(ctas) - min(ctas)) / 1e3,
                "barrier1_us": (s[1] - max(ctas)) / 1e3, "sum_gather_us": (s[2] - s[1]) / 1e3,
                "barrier2_us": (s[3] - s[2]) / 1e3, "total_us": (s[3] - s[0]) / 1e3}

    def check(self) -> None:
        s = int(self.status.item())
        if s:
            raise RuntimeError(f"fused tensor-parallel all-reduce failed (status {s}): "
                               + ("a peer did not arrive" if s >= 100 else "an on-chip pipeline wait timed out"))


class _FusedRowParallelFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w, helper):
        ctx.save_for_backward(y, w)
        return helper(y.to(torch.bfloat16), w.t().to(torch.bfloat16)).to(y.dtype)

    @staticmethod
    def backward(ctx, dout):
        y, w = ctx.saved_tensors
        d = dout.to(w.dtype)
        return d @ w.t(), y.t().to(w.dtype) @ d, None


def fused_row_parallel(y: torch.Tensor, w: torch.Tensor, helper: FusedRowParallel) -> torch.Tensor:
    """all_reduce(y @ w) over the helper's group with one fused kernel (y [T, K], w [K, N])."""
    return _FusedRowParallelFn.apply(y, w, helper)
