"""Native Sparse Attention block: compressed + selected + local branches with gates.

Parameter tree and the reference-compatible computation follow
``src/base_model/models/nsa.py:173-737``: ``q_proj/k_proj/v_proj/o_proj`` (no
bias), ``g_proj`` (3 sigmoid gates per head), ``norm1``/``norm2``, ``ff``; RoPE
on Q and K (``pe_type='rope'``; odd head dims fall back to sinusoidal input
encoding).

Branches:

1. compressed: K and V mean-pooled over blocks of ``block_size`` tokens; every
   query attends to the completed blocks; the block scores also rank blocks
   for branch 2;
2. selected: queries grouped by ``select_block`` tokens attend to the top
   ``block_counts`` selection blocks of their group (current block always
   included), causally;
3. local: causal attention over the last ``window_size`` tokens, or full causal
   attention when ``full_causal_window`` is set -- which is what the reference
   actually runs (``nsa.py:404-407``) and the default here, for checkpoint
   parity.

With ``select_block == block_size`` (the reference ties both to one message)
the computation is the reference's; larger selection blocks aggregate the
compressed scores of the compression blocks they contain.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .common import Dense, LayerNorm
from .rope import apply_rope, rotary_embedding, sinusoidal
from ..ops.attention import attention_probsum, flash_attention, flash_attention_lse, kernel_supported
from .transformer import FFN, causal_attention, effective_heads


class NSABlock(nn.Module):
    is_transformer = True

    def __init__(self, H, n_heads=16, d_ff=0, block_size=26, select_block=None, block_counts=16,
                 window_size=512, full_causal_window=True, dtype=torch.float32, max_cache_len=26000,
                 pe_type="rope", rope_base=10000.0, dropout=0.0, impl="torch"):
        super().__init__()
        self.H = H
        self.nh = effective_heads(H, n_heads)
        self.hd = H // self.nh
        self.block_size = block_size
        self.select_block = select_block or block_size
        if self.select_block % block_size:
            raise ValueError("select_block must be a multiple of block_size")
        self.block_counts = block_counts
        self.window = None if full_causal_window else window_size
        self.compute_dtype = dtype
        self.max_cache_len = max_cache_len
        self.pe = pe_type if not (pe_type == "rope" and self.hd % 2) else "sinusoidal"
        self.rope_base = rope_base
        self.impl = impl
        self.q_proj = Dense(H, H, bias=False)
        self.k_proj = Dense(H, H, bias=False)
        self.v_proj = Dense(H, H, bias=False)
        self.o_proj = Dense(H, H, bias=False)
        self.g_proj = Dense(H, self.nh * 3, bias=False)
        self.norm1 = LayerNorm(H)
        self.norm2 = LayerNorm(H)
        self.ff = FFN(H, d_ff or 4 * H)

    # -- branches -------------------------------------------------------------------
    def _compressed(self, q, k, v, scale, q_offset=0):
        """q (B,Lq,nh,hd), k/v (B,Lk,nh,hd) -> o (B,Lq,nh,hd), importance (B,Lq,nb)."""
        B, Lq, nh, hd = q.shape
        BS = self.block_size
        nb = k.shape[1] // BS
        kc = k[:, :nb * BS].reshape(B, nb, BS, nh, hd).float().mean(2)
        vc = v[:, :nb * BS].reshape(B, nb, BS, nh, hd).float().mean(2)
        t = torch.arange(q_offset, q_offset + Lq, device=q.device)
        if nb > 0 and kernel_supported(q, k, v):
            # flash kernels: compressed block n sits at its last token, (n + 1) * BS - 1
            kcb, vcb = kc.to(q.dtype), vc.to(q.dtype)
            kpos = ((torch.arange(nb, device=q.device) + 1) * BS - 1).to(torch.int32).expand(B, nb)
            o, lse = flash_attention_lse(q, kcb, vcb, scale, q_offset=q_offset, kpos=kpos)
            imp = attention_probsum(q, kcb, lse, scale, q_offset=q_offset, kpos=kpos)
            visible = torch.clamp((t - BS + 1) // BS + 1, min=0)
            cmask = torch.arange(nb, device=q.device)[None, :] < visible[:, None]
            cur = (t // BS)[:, None] == torch.arange(nb, device=q.device)[None, :]
            imp = torch.where(cur[None], torch.ones_like(imp), imp).masked_fill(~cmask[None], -1e9)
            return o, imp
        sc = torch.einsum("blhd,bnhd->blhn", q.float() * scale, kc)
        visible = torch.clamp((t - BS + 1) // BS + 1, min=0)
        cmask = torch.arange(nb, device=q.device)[None, :] < visible[:, None]      # (Lq, nb)
        sc = sc.masked_fill(~cmask[None, :, None, :], float("-inf"))
        attn = torch.softmax(sc, dim=-1).nan_to_num(0.0)
        attn = attn * (visible > 0)[None, :, None, None]
        o = torch.einsum("blhn,bnhd->blhd", attn, vc)
        imp = attn.sum(2)                                                            # (B, Lq, nb)
        cur = (t // BS)[:, None] == torch.arange(nb, device=q.device)[None, :]
        imp = torch.where(cur[None], torch.ones_like(imp), imp)
        imp = imp.masked_fill(~cmask[None], -1e9)
        return o.to(q.dtype), imp

    def _select(self, q, k, v, imp, scale, q_offset=0):
        """Top-S selection blocks per query group, causal attention over their tokens."""
        B, Lq, nh, hd = q.shape
        Lk = k.shape[1]
        SB, BS = self.select_block, self.block_size
        nsb = Lk // SB
        ratio = SB // BS
        # compression-block importance -> selection-block importance
        imp_s = imp[..., :nsb * ratio].reshape(B, Lq, nsb, ratio).max(-1).values if ratio > 1 else imp[..., :nsb]
        S = min(self.block_counts, max(nsb, 1))
        ng = (Lq + SB - 1) // SB
        pad = ng * SB - Lq
        impg = torch.nn.functional.pad(imp_s, (0, 0, 0, pad)).reshape(B, ng, SB, nsb).mean(2)
        top = impg.topk(S, dim=-1).indices.clamp(0, max(nsb - 1, 0))                # (B, ng, S)
        qg = torch.nn.functional.pad(q, (0, 0, 0, 0, 0, pad)).reshape(B, ng, SB, nh, hd)
        off = torch.arange(S * SB, device=q.device)
        kpos = top[..., off // SB] * SB + (off % SB)                                  # (B, ng, S*SB)
        if SB == 64 and nsb >= 1 and kernel_supported(q, k, v):
            # selection blocks of the kernels' key tile: read in place, no gathered copy
            from ..ops.attention import flash_attention_blocks
            qoff = (q_offset + torch.arange(ng, device=q.device) * SB).repeat(B)
            o = flash_attention_blocks(qg.reshape(B * ng, SB, nh, hd), k, v, top.reshape(B * ng, S),
                                       kpos.reshape(B * ng, S * SB), qoff, scale)
            return o.reshape(B, ng * SB, nh, hd)[:, :Lq]
        kb = k[:, :nsb * SB].reshape(B, nsb, SB, nh, hd)
        vb = v[:, :nsb * SB].reshape(B, nsb, SB, nh, hd)
        bidx = torch.arange(B, device=q.device)[:, None, None]
        ksel = kb[bidx, top].reshape(B, ng, S * SB, nh, hd)
        vsel = vb[bidx, top].reshape(B, ng, S * SB, nh, hd)
        if kernel_supported(q, k, v):
            # flash kernels over the gathered blocks: every (batch, group) is one batch entry
            qoff = (q_offset + torch.arange(ng, device=q.device) * SB).repeat(B)
            o = flash_attention(qg.reshape(B * ng, SB, nh, hd), ksel.reshape(B * ng, S * SB, nh, hd),
                                vsel.reshape(B * ng, S * SB, nh, hd), scale=scale,
                                kpos=kpos.reshape(B * ng, S * SB), qoff=qoff)
            return o.reshape(B, ng * SB, nh, hd)[:, :Lq]
        sc = torch.einsum("bgqhd,bgkhd->bgqhk", qg.float() * scale, ksel.float())
        qpos = q_offset + torch.arange(ng * SB, device=q.device).reshape(ng, SB)
        causal = kpos[:, :, None, :] <= qpos[None, :, :, None]                       # (B, ng, SB, S*SB)
        sc = sc.masked_fill(~causal[:, :, :, None, :], float("-inf"))
        attn = torch.softmax(sc, dim=-1).nan_to_num(0.0)
        o = torch.einsum("bgqhk,bgkhd->bgqhd", attn, vsel.float())
        return o.reshape(B, ng * SB, nh, hd)[:, :Lq].to(q.dtype)

    def _qkv(self, x, offset=0):
        B, L, H = x.shape
        cd = self.compute_dtype
        h = self.norm1(x)
        q = self.q_proj(h, cd).reshape(B, L, self.nh, self.hd)
        k = self.k_proj(h, cd).reshape(B, L, self.nh, self.hd)
        v = self.v_proj(h, cd).reshape(B, L, self.nh, self.hd)
        if self.pe == "rope":
            cos, sin = rotary_embedding(self.hd, L, self.rope_base, x.device, offset=offset)
            q, k = apply_rope(q, k, cos, sin)
        g = torch.sigmoid(self.g_proj(h, cd).float()).reshape(B, L, self.nh, 3)
        return q, k, v, g

    def _mix(self, x, q, k, v, g, q_offset=0):
        scale = self.hd ** -0.5
        o_cmp, imp = self._compressed(q, k, v, scale, q_offset)
        o_slc = self._select(q, k, v, imp, scale, q_offset)
        o_win = causal_attention(q, k, v, scale=scale, window=self.window, q_offset=q_offset)
        o = g[..., 0:1] * o_cmp.float() + g[..., 1:2] * o_slc.float() + g[..., 2:3] * o_win.float()
        B, L = o.shape[:2]
        x = x + self.o_proj(o.reshape(B, L, self.H).to(self.compute_dtype), self.compute_dtype).float()
        return x + self.ff(self.norm2(x), self.compute_dtype).float()

    def forward(self, x):
        B, L, H = x.shape
        if self.pe != "rope":
            x = x + sinusoidal(L, H, x.device)
        q, k, v, g = self._qkv(x)
        return self._mix(x, q, k, v, g)

    # -- decode: keep the full K/V cache; recompute branch outputs for the new tokens --
    def initial_state(self, batch, device=None):
        z = torch.zeros(batch, self.max_cache_len, self.nh, self.hd, dtype=self.compute_dtype, device=device)
        return (z, z.clone(), torch.zeros(batch, dtype=torch.long, device=device))

    def prefill(self, x, max_cache_len=None):
        B, L, H = x.shape
        out = self(x)
        xe = x + sinusoidal(L, H, x.device) if self.pe != "rope" else x
        _, k, v, _ = self._qkv(xe)
        st = self.initial_state(B, x.device)
        st[0][:, :L] = k.to(st[0].dtype)
        st[1][:, :L] = v.to(st[1].dtype)
        st[2].fill_(L)
        return st, out

    def step(self, state, x):
        kc, vc, pos = state
        B, L, H = x.shape
        p0 = int(pos[0])
        if self.pe != "rope":
            x = x + sinusoidal(L, H, x.device, offset=p0)
        q, k, v, g = self._qkv(x, offset=p0)
        kc[:, p0:p0 + L] = k.to(kc.dtype)
        vc[:, p0:p0 + L] = v.to(vc.dtype)
        keys, vals = kc[:, :p0 + L], vc[:, :p0 + L]
        return (kc, vc, pos + L), self._mix(x, q, keys, vals, g, q_offset=p0)
