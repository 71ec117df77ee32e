"""Pre-LN Transformer block (attention backbone and the hybrid's global mixer).

Same computation and parameter tree as the reference ``TransformerBlock``
(``src/base_model/models/transformer.py:114-392``): optional sinusoidal input
encoding, ``norm1 -> causal MHA -> residual``, ``norm2 -> ff (Dense, gelu,
Dense) -> residual``.  The attention projections keep Flax's
``MultiHeadDotProductAttention`` layout (``attn/{query,key,value}/kernel``
``(H, nh, hd)``, ``attn/out/kernel`` ``(nh, hd, H)``, biases included) and the
FFN keeps ``ff/layers_0`` and ``ff/layers_2``.

Decode uses a static KV cache ``(k (B,nh,max,hd), v, pos (B,))``; ``prefill``
runs the training forward and fills the cache, like the reference.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .common import Dense, LayerNorm, gelu_tanh, lecun_normal_
from .rope import sinusoidal, sinusoidal_at


def effective_heads(H: int, n_heads: int) -> int:
    while n_heads > 1 and H % n_heads:
        n_heads -= 1
    return n_heads


class HeadProj(nn.Module):
    """(H) -> (nh, hd) projection with Flax DenseGeneral parameter shapes."""

    def __init__(self, H, nh, hd):
        super().__init__()
        self.kernel = nn.Parameter(lecun_normal_(torch.empty(H, nh, hd), H))
        self.bias = nn.Parameter(torch.zeros(nh, hd))

    def forward(self, x, dtype=None):
        w = self.kernel if dtype is None else self.kernel.to(dtype)
        return torch.einsum("...d,dnk->...nk", x.to(w.dtype), w) + self.bias.to(w.dtype)


class OutProj(nn.Module):
    def __init__(self, nh, hd, H):
        super().__init__()
        self.kernel = nn.Parameter(lecun_normal_(torch.empty(nh, hd, H), nh * hd))
        self.bias = nn.Parameter(torch.zeros(H))

    def forward(self, o, dtype=None):
        w = self.kernel if dtype is None else self.kernel.to(dtype)
        return torch.einsum("...nk,nkd->...d", o.to(w.dtype), w) + self.bias.to(w.dtype)


class MHA(nn.Module):
    def __init__(self, H, nh):
        super().__init__()
        hd = H // nh
        self.query = HeadProj(H, nh, hd)
        self.key = HeadProj(H, nh, hd)
        self.value = HeadProj(H, nh, hd)
        self.out = OutProj(nh, hd, H)


class FFN(nn.Module):
    def __init__(self, H, d_ff):
        super().__init__()
        self.layers_0 = Dense(H, d_ff)
        self.layers_2 = Dense(d_ff, H)

    def forward(self, x, dtype=None):
        return self.layers_2(gelu_tanh(self.layers_0(x, dtype=dtype)), dtype=dtype)


def causal_attention(q, k, v, scale=None, window=None, q_offset: int = 0):
    """q (B, Lq, nh, hd), k/v (B, Lk, nh, hd) -> (B, Lq, nh, hd).

    Query i (absolute position q_offset + i) sees keys j <= position (and within
    ``window`` tokens when given).  The CUDA path is the sm_100a flash kernel when
    available; otherwise an exact blocked softmax in torch.
    """
    B, Lq, nh, hd = q.shape
    Lk = k.shape[1]
    scale = scale if scale is not None else hd ** -0.5
    if q.is_cuda:
        from ..ops.attention import flash_attention
        return flash_attention(q, k, v, scale=scale, causal=True, window=window, q_offset=q_offset)
    qh = q.transpose(1, 2).float() * scale
    kh = k.transpose(1, 2).float()
    vh = v.transpose(1, 2).float()
    out = torch.empty(B, nh, Lq, hd, dtype=torch.float32, device=q.device)
    blk = 1024
    kpos = torch.arange(Lk, device=q.device)
    for s in range(0, Lq, blk):
        e = min(Lq, s + blk)
        sc = qh[:, :, s:e] @ kh.transpose(-1, -2)
        qpos = torch.arange(q_offset + s, q_offset + e, device=q.device)[:, None]
        m = kpos[None, :] <= qpos
        if window is not None:
            m &= kpos[None, :] > qpos - window
        sc = sc.masked_fill(~m, float("-inf"))
        out[:, :, s:e] = torch.softmax(sc, dim=-1).nan_to_num(0.0) @ vh
    return out.transpose(1, 2).to(q.dtype)


class TransformerBlock(nn.Module):
    is_transformer = True

    def __init__(self, H, n_heads=16, d_ff=0, dtype=torch.float32, max_cache_len=26000,
                 use_positional_encoding=True, dropout=0.0, impl="torch"):
        super().__init__()
        self.H = H
        self.nh = effective_heads(H, n_heads)
        self.hd = H // self.nh
        self.d_ff = d_ff or 4 * H
        self.compute_dtype = dtype
        self.max_cache_len = max_cache_len
        self.use_pe = use_positional_encoding
        self.impl = impl
        self.attn = MHA(H, self.nh)
        self.norm1 = LayerNorm(H)
        self.norm2 = LayerNorm(H)
        self.ff = FFN(H, self.d_ff)

    def _qkv(self, h):
        cd = self.compute_dtype
        return (self.attn.query(h, cd), self.attn.key(h, cd), self.attn.value(h, cd))

    def forward(self, x):
        """x (B, L, H) -> (B, L, H)."""
        B, L, H = x.shape
        if self.use_pe:
            x = x + sinusoidal(L, H, x.device)
        h = self.norm1(x)
        q, k, v = self._qkv(h)
        o = causal_attention(q, k, v)
        x = x + self.attn.out(o, self.compute_dtype).float()
        return x + self.ff(self.norm2(x), self.compute_dtype).float()

    # -- decode -------------------------------------------------------------------
    def initial_state(self, batch, device=None):
        z = torch.zeros(batch, self.nh, self.max_cache_len, self.hd, dtype=self.compute_dtype, device=device)
        return (z, z.clone(), torch.zeros(batch, dtype=torch.long, device=device))

    def prefill(self, x, max_cache_len=None):
        out = self(x)
        B, L, H = x.shape
        xe = x + sinusoidal(L, H, x.device) if self.use_pe else x
        _, k, v = self._qkv(self.norm1(xe))
        st = self.initial_state(B, x.device)
        st[0][:, :, :L] = k.transpose(1, 2).to(st[0].dtype)
        st[1][:, :, :L] = v.transpose(1, 2).to(st[1].dtype)
        st[2].fill_(L)
        return st, out

    def step(self, state, x):
        kc, vc, pos = state
        B, L, H = x.shape
        p0 = int(pos[0])
        if self.use_pe:
            x = x + sinusoidal(L, H, x.device, offset=p0)
        h = self.norm1(x)
        q, k, v = self._qkv(h)
        kc[:, :, p0:p0 + L] = k.transpose(1, 2).to(kc.dtype)
        vc[:, :, p0:p0 + L] = v.transpose(1, 2).to(vc.dtype)
        keys = kc[:, :, :p0 + L].transpose(1, 2)
        vals = vc[:, :, :p0 + L].transpose(1, 2)
        o = causal_attention(q, keys, vals, q_offset=p0)
        x = x + self.attn.out(o, self.compute_dtype).float()
        x = x + self.ff(self.norm2(x), self.compute_dtype).float()
        return (kc, vc, pos + L), x
