"""Context (sequence) parallelism for the S5 layer.

Each rank of a context-parallel group holds one contiguous segment (length Ls) of every
sequence.  S5's state obeys the diagonal complex recurrence x_t = lam * x_{t-1} + Bu_t, so
a segment's states from an initial state x_in are its states from zero plus
lam^(t+1) * x_in (t = 0 .. Ls-1 within the segment), and the initial state of rank r is

    x_in[r] = sum_{j < r} x_loc[j] * lam^(Ls * (r - 1 - j)),

with x_loc[j] the final state of segment j from zero.  One all-gather of the local final
states (``torch.distributed.nn.functional.all_gather``, so the backward sums the state
gradients back onto their owners) carries the recurrence; the scan itself is the layer's
own (the ``s5_scan`` kernels on CUDA).  Parameters stay replicated and their gradients are
summed over the group like data-parallel gradients.  Bidirectional S5 layers need the
suffix as well and are not supported.  The reference's S5 layer is
``src/base_model/models/s5/ssm.py``; it has no context parallelism.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models.s5 import S5


class S5CP(nn.Module):
    def __init__(self, inner: S5, group=None):
        super().__init__()
        if inner.bidirectional:
            raise ValueError("a bidirectional S5 layer cannot run context-parallel")
        self.inner, self.group = inner, group

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        from torch.distributed.nn.functional import all_gather
        m, grp = self.inner, self.group
        r = dist.get_rank(grp)
        Ls = u.shape[1]
        lb, bb = m.discrete()
        Bu = torch.einsum("ph,blh->blp", bb, u.to(torch.complex64))
        xs, xl = m._scan(lb, Bu)
        allx = torch.stack(all_gather(torch.view_as_real(xl).contiguous(), group=grp), 0)     # (W, B, P, 2)
        allx = torch.view_as_complex(allx.contiguous())
        x_in = torch.zeros_like(xl)
        lam_seg = lb ** Ls
        for j in range(r):
            x_in = x_in * lam_seg + allx[j]
        x_in = x_in + 0.0 * allx.sum()             # every rank keeps the gather in its graph
        t = torch.arange(1, Ls + 1, device=u.device, dtype=torch.float32)
        pw = torch.exp(t[:, None] * torch.log(lb)[None, :])                                    # (Ls, P)
        xs = xs + pw[None] * x_in[:, None, :]
        y = torch.einsum("hp,blp->blh", m._C(), xs).real
        if m.conj_sym:
            y = 2 * y
        return y + m.D * u


def shard_s5_cp(model: nn.Module, group=None) -> nn.Module:
    """Wrap every ``S5`` layer of ``model`` for context parallelism."""
    for _, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, S5):
                setattr(mod, cname, S5CP(child, group))
    return model
