"""Causal (optionally windowed) attention on CUDA for the attention backbones.

Full causal attention runs through torch's fused scaled-dot-product attention;
a sliding window, or queries offset into a longer key sequence (decode), run
the exact blocked softmax below.  Both keep memory linear in the sequence.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _blocked(q, k, v, scale, window, q_offset, blk=2048):
    B, Lq, nh, hd = q.shape
    Lk = k.shape[1]
    qh = q.transpose(1, 2)
    kh = k.transpose(1, 2)
    vh = v.transpose(1, 2)
    out = torch.empty(B, nh, Lq, hd, dtype=q.dtype, device=q.device)
    kpos = torch.arange(Lk, device=q.device)
    for s in range(0, Lq, blk):
        e = min(Lq, s + blk)
        lo = 0 if window is None else max(0, q_offset + s - window + 1)
        hi = min(Lk, q_offset + e)
        qpos = torch.arange(q_offset + s, q_offset + e, device=q.device)[:, None]
        m = kpos[None, lo:hi] <= qpos
        if window is not None:
            m &= kpos[None, lo:hi] > qpos - window
        out[:, :, s:e] = F.scaled_dot_product_attention(qh[:, :, s:e], kh[:, :, lo:hi], vh[:, :, lo:hi],
                                                        attn_mask=m, scale=scale)
    return out.transpose(1, 2)


def flash_attention(q, k, v, scale=None, causal=True, window=None, q_offset=0):
    """q (B, Lq, nh, hd), k/v (B, Lk, nh, hd) -> (B, Lq, nh, hd)."""
    if window is None and q_offset == 0 and q.shape[1] == k.shape[1]:
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=causal, scale=scale)
        return o.transpose(1, 2)
    return _blocked(q, k, v, scale, window, q_offset)
