"""Context (sequence) parallelism for the attention backbones: transformer and NSA blocks.

Each rank of a context-parallel group holds one contiguous segment of every sequence (the
same split as ``Mamba3CP``: rank r holds positions [r * Ls, (r + 1) * Ls)).  Attention is
causal, so rank r needs the keys and values of segments 0 .. r: they are all-gathered
(``torch.distributed.nn.functional.all_gather``, whose backward sums the key / value
gradients back onto their owners) and the rank's queries attend with a query offset of
r * Ls -- the offset mode of the attention kernels (``csrc/attention.cu``).  Positional
encodings (sinusoidal or RoPE) are taken at the absolute positions.  Parameters stay
replicated; their gradients are summed over the group like data-parallel gradients.

The reference has no context parallelism for attention (its only sequence-parallel path is
the Mamba3 phase split, ``src/base_model/models/mamba3_seqpar.py``); the build plan asks for
it for the NSA + hybrid configuration.

NSA needs segments that start on a selection-block boundary (``Ls`` a multiple of the
selection block): its query groups and block top-k then match the full-sequence forward.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models.nsa import NSABlock
from ..models.rope import sinusoidal
from ..models.transformer import TransformerBlock, causal_attention


class _ContiguousGrad(torch.autograd.Function):
    """Identity whose backward hands on a contiguous gradient: the collective in the
    all-gather's backward reads its input buffers as dense memory, and a slice of the
    concatenated gradient along the sequence dimension is not."""

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return g.contiguous()


def gather_prefix(t: torch.Tensor, group=None, dim: int = 1) -> torch.Tensor:
    """Concatenate the segments of ranks 0 .. this rank along ``dim`` (autograd-aware)."""
    from torch.distributed.nn.functional import all_gather
    parts = all_gather(t.contiguous(), group=group)
    return torch.cat([_ContiguousGrad.apply(p) for p in parts[:dist.get_rank(group) + 1]], dim=dim)


class TransformerBlockCP(nn.Module):
    is_transformer = True

    def __init__(self, full: TransformerBlock, group=None):
        super().__init__()
        self.inner, self.group = full, group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = self.inner
        B, Ls, H = x.shape
        start = dist.get_rank(self.group) * Ls
        if m.use_pe:
            x = x + sinusoidal(Ls, H, x.device, offset=start)
        q, k, v = m._qkv(m.norm1(x))
        o = causal_attention(q, gather_prefix(k, self.group), gather_prefix(v, self.group), q_offset=start)
        x = x + m.attn.out(o, m.compute_dtype).float()
        return x + m.ff(m.norm2(x), m.compute_dtype).float()


class NSABlockCP(nn.Module):
    is_transformer = True

    def __init__(self, full: NSABlock, group=None):
        super().__init__()
        self.inner, self.group = full, group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = self.inner
        B, Ls, H = x.shape
        if Ls % m.select_block:
            raise ValueError(f"segment length {Ls} is not a multiple of the NSA selection block {m.select_block}")
        start = dist.get_rank(self.group) * Ls
        if m.pe != "rope":
            x = x + sinusoidal(Ls, H, x.device, offset=start)
        q, k, v, g = m._qkv(x, offset=start)
        return m._mix(x, q, gather_prefix(k, self.group), gather_prefix(v, self.group), g, q_offset=start)


def context_parallel_attention(model: nn.Module, group=None) -> nn.Module:
    """Replace every ``TransformerBlock`` and ``NSABlock`` of a model by its context-parallel
    wrapper (parameters shared with the original block)."""
    for _, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, NSABlock):
                setattr(mod, cname, NSABlockCP(child, group))
            elif isinstance(child, TransformerBlock):
                setattr(mod, cname, TransformerBlockCP(child, group))
    return model
