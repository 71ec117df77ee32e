"""Parameter-holding building blocks named like the reference's Flax modules.

Every parameter lives under the attribute path that the reference's Flax tree
uses (``Dense`` -> ``kernel``/``bias``, ``LayerNorm`` -> ``scale``/``bias``,
``Embed`` -> ``embedding``, ``RMSNorm`` -> ``scale``), so a module's
``named_parameters()`` maps one-to-one onto the reference checkpoint tree
(``docs/architecture.md:35-39`` of the reference).  Kernels are stored
``(in, out)`` as in Flax; parameters are float32.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


def lecun_normal_(t: torch.Tensor, fan_in: int, gen=None) -> torch.Tensor:
    # truncated normal (+-2 std) with variance 1/fan_in, like jax's lecun_normal
    std = math.sqrt(1.0 / fan_in) / 0.87962566103423978
    with torch.no_grad():
        t.normal_(0, 1, generator=gen)
        t.clamp_(-2, 2).mul_(std)
    return t


class Dense(nn.Module):
    def __init__(self, d_in: int, d_out: int, bias: bool = True):
        super().__init__()
        self.d_in, self.d_out = d_in, d_out
        self.kernel = nn.Parameter(lecun_normal_(torch.empty(d_in, d_out), d_in))
        self.bias = nn.Parameter(torch.zeros(d_out)) if bias else None

    def forward(self, x, dtype=None):
        if dtype == torch.bfloat16 and x.is_cuda and (self.d_in % 8 or self.d_out % 8):
            from ..ops.linear import linear_bf16      # aligned tensor-core path for odd widths
            return linear_bf16(x, self.kernel, self.bias).to(dtype)
        w = self.kernel if dtype is None else self.kernel.to(dtype)
        y = x.to(w.dtype) @ w
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y


class LayerNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d))
        self.bias = nn.Parameter(torch.zeros(d))

    def forward(self, x):
        return F.layer_norm(x.float(), (x.shape[-1],), self.scale, self.bias, self.eps)


class BatchNorm(nn.Module):
    """Batch normalisation over every axis but the last (the reference's ``--batchnorm``
    choice of ``SequenceLayer`` norm, ``src/base_model/models/layers.py:81-83``): batch
    statistics in training, averaged over the data-parallel ranks (the reference's
    ``axis_name='batch'``); running averages ``r = momentum * r + (1 - momentum) * batch``
    used in evaluation.  ``scale`` / ``bias`` carry the same names as ``LayerNorm``'s."""

    def __init__(self, d: int, momentum: float = 0.9, eps: float = 1e-5, group=None):
        super().__init__()
        self.momentum, self.eps, self.group = momentum, eps, group
        self.scale = nn.Parameter(torch.ones(d))
        self.bias = nn.Parameter(torch.zeros(d))
        self.register_buffer("mean", torch.zeros(d))
        self.register_buffer("var", torch.ones(d))

    def forward(self, x):
        xf = x.float()
        if self.training:
            dims = tuple(range(xf.dim() - 1))
            st = torch.cat([xf.mean(dims), (xf * xf).mean(dims)])
            import torch.distributed as dist
            if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
                from torch.distributed.nn.functional import all_reduce
                st = all_reduce(st, group=self.group) / dist.get_world_size(self.group)
            m, m2 = st.split(xf.shape[-1])
            var = (m2 - m * m).clamp_min(0.0)
            with torch.no_grad():
                self.mean.mul_(self.momentum).add_(m.detach(), alpha=1 - self.momentum)
                self.var.mul_(self.momentum).add_(var.detach(), alpha=1 - self.momentum)
        else:
            m, var = self.mean, self.var
        return (xf - m) * torch.rsqrt(var + self.eps) * self.scale + self.bias


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d))

    def forward(self, x):
        xf = x.float()
        return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.scale


class Embed(nn.Module):
    def __init__(self, n: int, d: int):
        super().__init__()
        # flax Embed default: variance_scaling(1, fan_in, normal, out_axis=0) -> std 1/sqrt(d)
        self.embedding = nn.Parameter(torch.randn(n, d) / math.sqrt(d))

    def forward(self, idx):
        if idx.is_cuda and self.embedding.dtype == torch.float32 and self.embedding.shape[1] % 4 == 0:
            return _EmbedGather.apply(idx.long().unsqueeze(-1), self.embedding)
        return self.embedding[idx]


class _EmbedGather(torch.autograd.Function):
    """Row gather of one or more tables summed (``csrc/embed.cu``: one warp per token in the
    forward, a vector-atomic scatter-add in the backward -- the sort-based dense embedding
    backward is two orders of magnitude slower for a 12k-row table and ~10^5 lookups)."""

    @staticmethod
    def forward(ctx, idx, *weights):
        from ..ops._ext import ext
        idx = idx.contiguous()          # a context-parallel segment is a strided view
        ctx.save_for_backward(idx)
        ctx.shapes = [w.shape for w in weights]
        return ext().embed_sum_fwd([w.contiguous() for w in weights], idx)

    @staticmethod
    def backward(ctx, g):
        from ..ops._ext import ext
        (idx,) = ctx.saved_tensors
        gws = [torch.zeros(s, dtype=torch.float32, device=g.device) for s in ctx.shapes]
        ext().embed_sum_bwd(gws, g.float().contiguous(), idx)
        return (None,) + tuple(gws)


def embed_sum(idx: torch.Tensor, weights) -> torch.Tensor:
    """``sum_f weights[f][idx[..., f]]`` (CUDA kernel for fp32 tables on the GPU)."""
    weights = list(weights)
    if idx.is_cuda and all(w.dtype == torch.float32 for w in weights) and weights[0].shape[1] % 4 == 0:
        return _EmbedGather.apply(idx.long(), *weights)
    out = weights[0][idx[..., 0]]
    for f in range(1, len(weights)):
        out = out + weights[f][idx[..., f]]
    return out


def gelu_tanh(x):
    return F.gelu(x, approximate="tanh")
