"""Context (sequence) parallelism for the Mamba3 mixer.

Each rank of a context-parallel group holds one contiguous segment of every
sequence.  The recurrence crosses segment boundaries through the same carry as
decoding: the angle state, the SSM state, and the previous token's rotated key
and value (the trapezoid rule couples a token to its predecessor).  The
reference only has a test-time version of this for phases 4-6
(``src/base_model/models/mamba3_seqpar.py:45-110``, all-gathered carry); here
the whole mixer runs segment-parallel with autograd:

1. every rank sums its segment's angle increments; an all-gather and an
   exclusive prefix give each rank its starting angle (mod 2 pi);
2. with absolute angles known, each rank runs its segment from a zero SSM state
   and obtains its local final state ``S_loc``, its total decay ``Delta`` and
   its last rotated key / value; one all-gather shares them;
3. the boundary recurrence ``S_end[r] = Delta[r] * (S_end[r-1] + c[r]) + S_loc[r]``
   (``c[r]`` = the trapezoid coupling of rank r's first token with rank r-1's
   last one) is solved by a prefix over ranks, giving rank r's initial state;
4. the segment is re-run from that initial state (the correction is linear in
   it; re-running keeps the code on the tested chunked path).

All collectives are ``torch.distributed.nn.functional.all_gather`` (gradients
flow back through reduce-scatter), so the backward pass is exact too.

On CUDA (the module's ``impl == "cuda"`` geometry) steps 2 and 4 are the tcgen05 chunk
walkers continued from a carried state and angle (``ops.mamba3_layer.mamba3_ssd_carry``):
each pass is one forward kernel and, in the backward, one reverse kernel whose initial
carry is the final-state gradient; the per-token prep, the boundary terms and the
recurrence over ranks stay small torch expressions.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..models.mamba3 import Mamba3
from ..ops.reference import mamba3_ref as ref

TWO_PI = 2.0 * math.pi


def _gather(x: torch.Tensor, group) -> torch.Tensor:
    from torch.distributed.nn.functional import all_gather
    return torch.stack(all_gather(x.contiguous(), group=group), 0)


class Mamba3CP(nn.Module):
    is_transformer = False

    def __init__(self, inner: Mamba3, group=None):
        super().__init__()
        self.inner = inner           # full (replicated) parameters
        self.group = group

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        if self.inner._cuda_ok(u):
            return self._forward_cuda(u)
        m, d = self.inner, self.inner.dims
        W = dist.get_world_size(self.group)
        r = dist.get_rank(self.group)
        nh = d.n_heads
        proj = m.in_proj(u, dtype=m.compute_dtype)
        z, x, B, C, ADT, DT, trap, ang = m._prep(proj)
        Bh = B[:, :, None, :].expand(-1, -1, nh, -1)
        Ch = C[:, :, None, :].expand(-1, -1, nh, -1)
        ADTt, DTt, trt = ADT.transpose(1, 2), DT.transpose(1, 2), trap.transpose(1, 2)
        # 1. starting angles (one all-gather)
        rate = torch.tanh(ang)[:, :, None, :] * math.pi * DTt.transpose(1, 2)[..., None]   # (Bt, L, H, R)
        sums = _gather(rate.sum(1), self.group)                                           # (W, Bt, H, R)
        off = sums[:r].sum(0) if r > 0 else torch.zeros_like(sums[0])
        off = off - TWO_PI * torch.floor(off / TWO_PI)
        # 2. local pass from zero state
        _, S_loc, angs, k_last, _ = ref.mamba3_ssd_chunked(
            Ch, Bh, x, ADTt, DTt, trt, ang, m.C_bias, m.B_bias, m.D, z, chunk_size=d.chunk_size,
            return_final_state="all", angle_offset=off)
        v_last = x[:, -1]                                                                  # (Bt, H, P)
        delta = torch.exp(ADTt.sum(-1))                                                    # (Bt, H)
        # coupling of this segment's first token with the previous segment's last token
        sig0 = torch.sigmoid(trt[:, :, 0])
        w0 = (1.0 - sig0) * DTt[:, :, 0]                                                   # (Bt, H)
        # one packed all-gather of every rank's boundary quantities
        Bt, H, P, N = S_loc.shape
        parts = [S_loc.reshape(Bt, H, -1), delta[..., None], k_last, v_last, w0[..., None]]
        sizes = [p.shape[-1] for p in parts]
        allp = _gather(torch.cat(parts, -1), self.group)                                 # (W, Bt, H, sum)
        allS, allD, allK, allV, allw = torch.split(allp, sizes, -1)
        allS = allS.reshape(W, Bt, H, P, N)
        allD, allw = allD[..., 0], allw[..., 0]
        # 3. boundary recurrence over ranks 0..r-1
        S_end = torch.zeros_like(S_loc)
        for k in range(r):
            c = torch.zeros_like(S_loc) if k == 0 else \
                allw[k][..., None, None] * allV[k - 1][..., :, None] * allK[k - 1][..., None, :]
            S_end = allD[k][..., None, None] * (S_end + c) + allS[k]
        if r > 0:
            S_init = S_end + w0[..., None, None] * allV[r - 1][..., :, None] * allK[r - 1][..., None, :]
        else:
            S_init = torch.zeros_like(S_loc)
        # every rank keeps both gathers in its graph (zero-weighted where unused), so the
        # backward reduce-scatters run on all ranks in the same order
        S_init = S_init + 0.0 * (allp.sum() + sums.sum())
        # 4. the segment from its true initial state
        y = ref.mamba3_ssd_chunked(Ch, Bh, x, ADTt, DTt, trt, ang, m.C_bias, m.B_bias, m.D, z,
                                   chunk_size=d.chunk_size, initial_state=S_init, angle_offset=off)
        return m._post(y)

    def _forward_cuda(self, u: torch.Tensor) -> torch.Tensor:
        from ..ops.mamba3_layer import mamba3_ssd_carry
        m, d = self.inner, self.inner.dims
        W = dist.get_world_size(self.group)
        r = dist.get_rank(self.group)
        Bt, L, Hm = u.shape
        nh, P, N, R = d.n_heads, d.headdim, d.d_state, d.R
        proj = m.in_proj(u, dtype=torch.bfloat16).reshape(Bt * L, -1)
        ldp = (d.d_in_proj + 7) // 8 * 8
        if ldp != d.d_in_proj:
            proj = F.pad(proj, (0, ldp - d.d_in_proj))
        proj = proj.contiguous()
        z, x, Bc, Cc, dd_dt, dd_A, trap, ang = m.split_proj(proj[:, :d.d_in_proj].float().view(Bt, L, -1))
        DT = F.softplus(dd_dt + m.dt_bias)                                                # (Bt, L, nh)
        A = torch.clamp(-F.softplus(dd_A), max=-m.A_floor)
        rate = torch.tanh(ang) * math.pi                                                   # (Bt, L, R)
        # 1. starting angles
        tot = torch.einsum("blr,blh->bhr", rate, DT)                                      # (Bt, nh, R)
        sums = _gather(tot, self.group)
        off = sums[:r].sum(0) if r > 0 else torch.zeros_like(tot)
        off = off - TWO_PI * torch.floor(off / TWO_PI)
        # 2. local pass from a zero state
        _, S_loc = mamba3_ssd_carry(proj, m, Bt, L, None, off)                             # (Bt, nh, P, N)
        delta = torch.exp((A * DT).sum(1))                                                 # (Bt, nh)
        th_last = off + tot
        Kb = m.B_norm(Bc[:, -1])[:, None, :] + m.B_bias[None]                             # (Bt, nh, N)
        k_last = ref.apply_rope(Kb, torch.cos(th_last), torch.sin(th_last))
        v_last = x[:, -1].reshape(Bt, nh, P)
        w0 = (1.0 - torch.sigmoid(trap[:, 0])) * DT[:, 0]                                 # (Bt, nh)
        parts = [S_loc.reshape(Bt, nh, -1), delta[..., None], k_last, v_last, w0[..., None]]
        sizes = [p.shape[-1] for p in parts]
        allp = _gather(torch.cat(parts, -1), self.group)
        allS, allD, allK, allV, allw = torch.split(allp, sizes, -1)
        allS = allS.reshape(W, Bt, nh, P, N)
        allD, allw = allD[..., 0], allw[..., 0]
        # 3. boundary recurrence over ranks 0..r-1
        S_end = torch.zeros_like(S_loc)
        for k in range(r):
            c = torch.zeros_like(S_loc) if k == 0 else \
                allw[k][..., None, None] * allV[k - 1][..., :, None] * allK[k - 1][..., None, :]
            S_end = allD[k][..., None, None] * (S_end + c) + allS[k]
        if r > 0:
            S_init = S_end + w0[..., None, None] * allV[r - 1][..., :, None] * allK[r - 1][..., None, :]
        else:
            S_init = torch.zeros_like(S_loc)
        S_init = S_init + 0.0 * (allp.sum() + sums.sum())
        # 4. the segment from its true initial state
        y, _ = mamba3_ssd_carry(proj, m, Bt, L, S_init.contiguous(), off.contiguous())
        return m._post(y.view(Bt, L, nh, P))


def shard_model_cp(model: nn.Module, group=None) -> nn.Module:
    """Wrap every ``Mamba3`` mixer, ``GDN`` mixer, ``S5`` layer and transformer / NSA block
    of ``model`` for context parallelism (the hybrid backbones mix them)."""
    from .cp_attention import context_parallel_attention
    from .cp_gdn import shard_gdn_cp
    from .cp_s5 import shard_s5_cp
    for _, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, Mamba3):
                setattr(mod, cname, Mamba3CP(child, group))
    return context_parallel_attention(shard_s5_cp(shard_gdn_cp(model, group), group), group)


def split_sequence(x: torch.Tensor, group=None, dim: int = 1) -> torch.Tensor:
    """This rank's contiguous segment of ``x`` along ``dim`` (length divisible by the group size)."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    n = x.shape[dim]
    if n % W:
        raise ValueError(f"sequence length {n} does not split over {W} context-parallel ranks")
    return x.narrow(dim, r * (n // W), n // W)
