"""Fused decoder + cross-entropy without materialising float32 logits.

The reference computes ``log_softmax(decoder(h))`` in float32 over the whole
sequence and picks the label column (``training/train_helpers.py:742-783``);
at 88k tokens x 12,288 classes that is 4.3 GB of float32 logits.  Here the
decoder GEMM runs over row chunks in bf16, the CE kernel turns each chunk's
logits into per-row losses and, in place, into ``w_t * (softmax - onehot)``;
the chunk's input and weight gradients are accumulated immediately.  The
training loss is a weighted mean, so its gradient is known in the forward
pass: backward only rescales the stored gradients by the upstream scalar.
"""
from __future__ import annotations

import torch

from ._ext import ext
from . import gemm as G
from . import weights as W

CHUNK_ROWS = 8192


class _LinearCEMean(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, kernel, bias, labels, weights):
        C = ext()
        shp = labels.shape
        d = h.shape[-1]
        V = kernel.shape[1]
        hf = h.reshape(-1, d).to(torch.bfloat16).contiguous()
        lab = labels.reshape(-1).contiguous()
        wr = weights.reshape(-1).float().contiguous()
        wk = W.bf16(kernel)
        T = hf.shape[0]
        loss_rows = torch.empty(T, dtype=torch.float32, device=h.device)
        dh = torch.empty_like(hf)
        dW = torch.zeros(d, V, dtype=torch.float32, device=h.device)
        db = torch.zeros(V, dtype=torch.float32, device=h.device)
        tc = G.USE_TC and V % 8 == 0 and d % 8 == 0
        for s in range(0, T, CHUNK_ROWS):
            e = min(T, s + CHUNK_ROWS)
            logits = G.mm(hf[s:e], wk) if tc else hf[s:e] @ wk
            loss_rows[s:e] = C.ce_fwd_bwd(logits, bias, lab[s:e], wr[s:e], V)
            if tc:
                dh[s:e] = G.mm_nt(logits, wk)
                G.mm_tn_acc(hf[s:e], logits, dW)          # fp32 accumulation across chunks
            else:
                dh[s:e] = logits @ wk.t()
                dW += torch.mm(hf[s:e].t(), logits, out_dtype=torch.float32)
            db += logits.sum(0, dtype=torch.float32)
        loss = (loss_rows * wr).sum()
        ctx.save_for_backward(dh, dW, db)
        ctx.shape, ctx.h_dtype = h.shape, h.dtype
        ctx.mark_non_differentiable(loss_rows)
        return loss, loss_rows.view(shp)

    @staticmethod
    def backward(ctx, gloss, _grows):
        dh, dW, db = ctx.saved_tensors
        return (dh.view(ctx.shape).to(ctx.h_dtype) * gloss, dW * gloss, db * gloss, None, None)


def linear_cross_entropy_mean(h, kernel, bias, labels, weights):
    """Returns (sum_t w_t * ce_t, per-token ce).  ``weights`` sum to 1 for a mean."""
    return _LinearCEMean.apply(h, kernel, bias, labels, weights)
