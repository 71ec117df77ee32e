"""Tensor parallelism for the Mamba3 mixer (heads split over a tensor-parallel group).

The reference splits Mamba3 heads over the ``tp`` mesh axis, computes the
projection for the rank's heads, normalises ``out_norm`` with a psum of the
sum of squares, and reduces the row-parallel ``out_proj`` with a psum
(``src/base_model/models/mamba3.py:209-233``).  Here:

* ``Mamba3TP`` holds the rank's slices of a full ``Mamba3``'s parameters:
  in_proj columns of its heads' ``z``/``x``/``dd_dt``/``dd_A``/``trap`` plus the
  shared ``B``/``C``/angle columns; per-head ``dt_bias``/``B_bias``/``C_bias``/``D``;
  its rows of ``out_norm``/``out_proj``;
* collectives are the two conjugate operators of tensor parallelism: the input
  enters through ``copy_to_tp`` (identity forward, gradient all-reduce) and the
  row-parallel output leaves through ``reduce_from_tp`` (all-reduce forward,
  identity backward); the RMS statistic is an all-reduce in both directions.

``shard_model(model, group)`` replaces every ``Mamba3`` mixer of a model in place,
keeping the rank's parameter slices (so per-rank optimizer state shrinks by the
TP degree for the mixer weights).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..models.mamba3 import Mamba3
from ..ops.reference import mamba3_ref as ref


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _AllReduceBoth(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def copy_to_tp(x, group):
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x, group):
    return _ReduceFromTP.apply(x, group)


def all_reduce_both(x, group):
    return _AllReduceBoth.apply(x, group)


class Mamba3TP(nn.Module):
    is_transformer = False

    def __init__(self, full: Mamba3, group=None):
        super().__init__()
        self.group = group
        T = dist.get_world_size(group)
        r = dist.get_rank(group)
        d = full.dims
        if d.n_heads % T:
            raise ValueError(f"{d.n_heads} heads do not split over tensor-parallel size {T}")
        self.full_dims = d
        self.tp, self.rank = T, r
        nhl = d.n_heads // T
        self.nhl, self.h0 = nhl, r * nhl
        P, N, nh, di = d.headdim, d.d_state, d.n_heads, d.d_inner
        hp = slice(self.h0 * P, (self.h0 + nhl) * P)
        hh = slice(self.h0, self.h0 + nhl)
        W = full.in_proj.kernel.detach()
        o_z, o_x, o_B, o_C = 0, di, 2 * di, 2 * di + N
        o_dt, o_A, o_tr, o_ang = o_C + N, o_C + N + nh, o_C + N + 2 * nh, o_C + N + 3 * nh
        head_cols = torch.cat([torch.arange(o_z, o_z + di)[hp], torch.arange(o_x, o_x + di)[hp],
                               torch.arange(o_dt, o_dt + nh)[hh], torch.arange(o_A, o_A + nh)[hh],
                               torch.arange(o_tr, o_tr + nh)[hh]])
        shared_cols = torch.cat([torch.arange(o_B, o_B + N), torch.arange(o_C, o_C + N),
                                 torch.arange(o_ang, o_ang + d.R)])
        self.register_buffer("_head_cols", head_cols, persistent=False)
        self.register_buffer("_shared_cols", shared_cols, persistent=False)
        self.in_proj_heads = nn.Parameter(W[:, head_cols].clone())
        self.in_proj_shared = nn.Parameter(W[:, shared_cols].clone())   # replicated on every TP rank
        self.dt_bias = nn.Parameter(full.dt_bias.detach()[hh].clone())
        self.B_bias = nn.Parameter(full.B_bias.detach()[hh].clone())
        self.C_bias = nn.Parameter(full.C_bias.detach()[hh].clone())
        self.D = nn.Parameter(full.D.detach()[hh].clone())
        self.B_norm_scale = nn.Parameter(full.B_norm.scale.detach().clone())
        self.C_norm_scale = nn.Parameter(full.C_norm.scale.detach().clone())
        self.out_norm_scale = nn.Parameter(full.out_norm.scale.detach()[hp].clone())
        self.out_proj_kernel = nn.Parameter(full.out_proj.kernel.detach()[hp].clone())
        self.A_floor = full.A_floor
        self.eps = 1e-6
        self.fused_out = None

    def _rms(self, x, scale):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + self.eps) * scale

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        """Head-parallel columns see the input through ``copy_to_tp``; the replicated
        B/C/angle columns are computed from the raw input and their (normalised)
        outputs pass through ``copy_to_tp``, so the replicated weights receive the
        full gradient on every rank and the input gradient is counted once."""
        d, nhl = self.full_dims, self.nhl
        P, N = d.headdim, d.d_state
        lead = u.shape[:-1]
        proj = copy_to_tp(u, self.group).float() @ self.in_proj_heads
        z, x, dd_dt, dd_A, trap = torch.split(proj, [nhl * P, nhl * P, nhl, nhl, nhl], -1)
        sh = u.float() @ self.in_proj_shared
        B, C, ang = torch.split(sh, [N, N, d.R], -1)
        shared = copy_to_tp(torch.cat([self._rms(B, self.B_norm_scale), self._rms(C, self.C_norm_scale), ang], -1),
                            self.group)
        B, C, ang = torch.split(shared, [N, N, d.R], -1)
        z = z.reshape(*lead, nhl, P)
        x = x.reshape(*lead, nhl, P)
        A = torch.clamp(-F.softplus(dd_A), max=-self.A_floor)
        DT = F.softplus(dd_dt + self.dt_bias)
        Bh = B[:, :, None, :].expand(-1, -1, nhl, -1)
        Ch = C[:, :, None, :].expand(-1, -1, nhl, -1)
        y = ref.mamba3_ssd_chunked(Ch, Bh, x, (A * DT).transpose(1, 2), DT.transpose(1, 2), trap.transpose(1, 2),
                                   ang, self.C_bias, self.B_bias, self.D, z, chunk_size=d.chunk_size)
        y = y.reshape(*lead, nhl * P)
        ss = all_reduce_both((y * y).sum(-1, keepdim=True), self.group)      # full-width RMS statistic
        yn = y * torch.rsqrt(ss / d.d_inner + self.eps) * self.out_norm_scale
        if self.fused_out is not None and yn.is_cuda and yn.numel() // yn.shape[-1] <= self.fused_out.M:
            from .tp_fused import fused_row_parallel
            out = fused_row_parallel(yn.reshape(-1, yn.shape[-1]), self.out_proj_kernel, self.fused_out)
            return out.reshape(*lead, -1).to(u.dtype)
        return reduce_from_tp(yn @ self.out_proj_kernel, self.group).to(u.dtype)

    def use_fused_out_proj(self, max_rows: int) -> None:
        """Route out_proj + its all-reduce through the fused peer-memory kernel
        (``parallel/tp_fused.py``) for inputs of up to ``max_rows`` tokens."""
        from .tp_fused import FusedRowParallel
        self.fused_out = FusedRowParallel(max_rows, self.out_proj_kernel.shape[1], self.group,
                                          self.out_proj_kernel.device)

    def tp_sharded_parameters(self) -> list:
        """This rank's head slices (the B / C / angle columns and BCNorm scales are replicated)."""
        return [self.in_proj_heads, self.dt_bias, self.B_bias, self.C_bias, self.D, self.out_norm_scale,
                self.out_proj_kernel]

    def full_in_proj_grad(self):
        """This rank's in_proj gradient scattered into the full (H, d_in_proj) layout."""
        g = torch.zeros(self.in_proj_heads.shape[0], self.full_dims.d_in_proj, dtype=self.in_proj_heads.grad.dtype)
        g[:, self._head_cols] = self.in_proj_heads.grad
        g[:, self._shared_cols] = self.in_proj_shared.grad
        return g


def shard_model(model: nn.Module, group=None) -> nn.Module:
    """Replace every ``Mamba3`` sub-module by its tensor-parallel slice (one whose head count
    does not divide over the group stays whole and replicated)."""
    T = dist.get_world_size(group)
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, Mamba3) and child.dims.n_heads % T:
                continue
            if isinstance(child, Mamba3):
                setattr(mod, cname, Mamba3TP(child, group))
    return model
