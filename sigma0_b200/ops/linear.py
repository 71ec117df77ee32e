"""bf16 tensor-core linear layer for widths that are not multiples of 8.

``y = x @ W + b`` with the bf16 shadow of ``W`` (fp32 master) and ``K`` padded to a
multiple of 8 so every GEMM operand row is 16-byte aligned (unaligned rows push
cuBLAS onto its slow byte-aligned kernels, or onto fp32 SIMT kernels when the
operands are fp32).  Output fp32; the weight gradient is returned in fp32 for the
flat gradient buffer.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import weights as W


def _pad(n: int) -> int:
    return (n + 7) // 8 * 8


class _LinearBf16(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kernel, bias):
        lead, K = x.shape[:-1], x.shape[-1]
        Kp = _pad(K)
        N = kernel.shape[1]
        Np = _pad(N)
        x2 = x.reshape(-1, K).to(torch.bfloat16)
        w = W.bf16(kernel)
        if Kp != K or Np != N:
            x2 = F.pad(x2, (0, Kp - K)) if Kp != K else x2
            w = F.pad(w, (0, Np - N, 0, Kp - K))
        y = (x2 @ w)
        if Np != N:
            y = y[:, :N]
        y = y.float()
        if bias is not None:
            y = y + bias
        ctx.save_for_backward(x2, w)
        ctx.K, ctx.N, ctx.lead, ctx.has_bias, ctx.xdtype = K, N, lead, bias is not None, x.dtype
        return y.reshape(*lead, -1)

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        g2 = g.reshape(-1, g.shape[-1])
        gb = g2.to(torch.bfloat16)
        Np = w.shape[1]
        if Np != ctx.N:
            gb = F.pad(gb, (0, Np - ctx.N))
        dx = (gb @ w.t())[:, :ctx.K].to(ctx.xdtype).reshape(*ctx.lead, ctx.K)
        dw = (x2.t() @ gb)[:ctx.K, :ctx.N].float()
        db = g2.float().sum(0) if ctx.has_bias else None
        return dx, dw, db


def linear_bf16(x, kernel, bias=None):
    return _LinearBf16.apply(x, kernel, bias)
