"""Context (sequence) parallelism for the GDN / KDA mixer.

Each rank of a context-parallel group holds one contiguous segment of every sequence.  The
gated delta rule carries a state S [hvd, hd] per head across segment boundaries, and every
chunk updates it affinely, S -> S M_c + N_c with M_c = diag(tot_c) - kc_c^T kd_c (see
``gated_delta_chunked(..., return_transition=True)``).  So a segment maps its initial state
S0 to S0 T + S_loc, where T is the product of its chunk transitions and S_loc its final
state from a zero start.  The mixer then runs in four steps:

1. the causal depthwise convolutions read the last ``kernel - 1`` pre-convolution rows of
   the previous segment (one all-gather of every rank's tail rows);
2. each rank runs its segment from a zero state and gets S_loc and T;
3. one all-gather of (S_loc, T); rank r composes S_in[r] = (...(S_loc[0] T[1] + S_loc[1]) ...)
   over the ranks before it;
4. the segment is re-run from S_in[r] (on CUDA through the chunk-scan kernels, which take
   an initial state and return its gradient).

All collectives are ``torch.distributed.nn.functional.all_gather`` (their backward sums the
gradients back onto the owning ranks), every rank keeps every gather in its graph so the
backward collectives run in the same order on all ranks, and the parameters stay replicated
(their gradients are summed over the group like data-parallel gradients).  The reference
has no GDN context parallelism; its build plan asks for the context-parallel state carry of
Mamba3 / GDN.  Here the carry goes through NCCL all-gathers, not through peer stores inside
the scan kernel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..models.gdn import GDN, gated_delta_chunked, l2_normalize


def _gather(t: torch.Tensor, group) -> torch.Tensor:
    from torch.distributed.nn.functional import all_gather
    return torch.stack(all_gather(t.contiguous(), group=group), 0)


class GDNCP(nn.Module):
    is_transformer = False

    def __init__(self, inner: GDN, group=None):
        super().__init__()
        self.inner, self.group = inner, group

    def _inputs(self, x: torch.Tensor):
        m, grp = self.inner, self.group
        B, L, _ = x.shape
        nh, hd, hvd = m.nh, m.hd, m.hvd
        q, k, v = m.q_proj(x), m.k_proj(x), m.v_proj(x)
        if m.use_conv:
            r = dist.get_rank(grp)
            kk = m.q_conv.k - 1
            tails = _gather(torch.cat([q[:, -kk:], k[:, -kk:], v[:, -kk:]], -1), grp)    # (W, B, kk, sum C)
            prev = tails[r - 1] if r > 0 else torch.zeros_like(tails[0])
            prev = prev + 0.0 * tails.sum()             # every rank keeps the gather in its graph
            pq, pk, pv = torch.split(prev, [q.shape[-1], k.shape[-1], v.shape[-1]], -1)
            q = F.silu(m.q_conv._conv(torch.cat([pq, q], 1)))
            k = F.silu(m.k_conv._conv(torch.cat([pk, k], 1)))
            v = F.silu(m.v_conv._conv(torch.cat([pv, v], 1)))
        q = l2_normalize(q.reshape(B, L, nh, hd)) * hd ** -0.5
        k = l2_normalize(k.reshape(B, L, nh, hd))
        v = v.reshape(B, L, nh, hvd)
        beta = torch.sigmoid(m.b_proj(x))
        alog = F.logsigmoid(m.gk_proj(x)).reshape(B, L, nh, hd if m.use_kda else 1)
        g = F.silu(m.g_proj(x)).reshape(B, L, nh, hvd)
        return q, k, v, beta, alog, g

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m, grp = self.inner, self.group
        r = dist.get_rank(grp)
        q, k, v, beta, alog, g = self._inputs(x)
        o0, S_loc, T = gated_delta_chunked(q, k, v, beta, alog, m.chunk, return_transition=True)
        allS, allT = _gather(S_loc, grp), _gather(T, grp)
        S_in = torch.zeros_like(S_loc)
        for j in range(r):
            S_in = S_in @ allT[j] + allS[j]
        S_in = S_in + 0.0 * (allS.sum() + allT.sum())
        o = o0 if r == 0 else gated_delta_chunked(q, k, v, beta, alog, m.chunk, S0=S_in)[0]
        if r == 0:
            o = o + 0.0 * S_in.sum()
        return m._out(x, o, g)


def shard_gdn_cp(model: nn.Module, group=None) -> nn.Module:
    """Wrap every ``GDN`` mixer of ``model`` for context parallelism."""
    for _, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, GDN):
                setattr(mod, cname, GDNCP(child, group))
    return model
