"""Causal (optionally windowed) attention on CUDA for the attention backbones.

Sliding-window attention and queries offset into a longer key sequence (decode, NSA
window branch), in bf16 with head dim 64 or 128, run the sm_100a flash kernels of
``csrc/attention.cu`` (forward and backward) -- the replacement for the
reference's cuDNN flash attention (``src/base_model/models/nsa.py:27-59``) and its
Pallas MHA (``src/base_model/models/transformer.py:19-85``).  Full causal attention takes torch's
fused attention; other dtypes / head sizes an exact blocked softmax in torch (memory
linear in the sequence).  ``flash_attention(..., force_kernel=True)`` runs the kernels
for the full causal case too (tests, benchmarks).
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


def _kernel_ready(t: torch.Tensor) -> torch.Tensor:
    """The kernels take strided [B, L, nh, hd] views whose strides are multiples of 8
    elements with a contiguous head dim and a 16-byte aligned base."""
    ok = (t.stride(3) == 1 and t.stride(0) % 8 == 0 and t.stride(1) % 8 == 0 and t.stride(2) % 8 == 0
          and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, window, q_offset, kpos, qoff):
        from ._ext import ext
        q, k, v = _kernel_ready(q), _kernel_ready(k), _kernel_ready(v)
        B, Lq, nh, hd = q.shape
        o = torch.empty_like(q, memory_format=torch.contiguous_format)
        lse = torch.empty(B, nh, Lq, dtype=torch.float32, device=q.device)
        ext().attn_fwd(q, k, v, o, lse, scale, window, q_offset, kpos, qoff)
        ctx.save_for_backward(q, k, v, o, lse, kpos, qoff)
        ctx.args = (scale, window, q_offset)
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, do, _dlse):
        from ._ext import ext
        q, k, v, o, lse, kpos, qoff = ctx.saved_tensors
        scale, window, q_offset = ctx.args
        do = _kernel_ready(do.to(torch.bfloat16))
        D = torch.empty_like(lse)
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        dk = torch.empty(k.shape, dtype=torch.bfloat16, device=k.device)
        dv = torch.empty(v.shape, dtype=torch.bfloat16, device=v.device)
        ext().attn_bwd(q, k, v, o, lse, do, D, dq, dk, dv, scale, window, q_offset, kpos, qoff)
        return dq.to(torch.bfloat16), dk, dv, None, None, None, None, None


class _FlashAttnSel(torch.autograd.Function):
    """Attention of query groups over block-indirect keys (``attn_sel_fwd`` / ``attn_sel_bwd``):
    the selected key / value blocks are read in place, and their gradients are added back into
    source-shaped fp32 buffers by the kernel."""

    @staticmethod
    def forward(ctx, q, k, v, kblk, kpos, qoff, scale):
        from ._ext import ext
        q, k, v = _kernel_ready(q), _kernel_ready(k), _kernel_ready(v)
        E, Lq, nh, hd = q.shape
        o = torch.empty_like(q, memory_format=torch.contiguous_format)
        lse = torch.empty(E, nh, Lq, dtype=torch.float32, device=q.device)
        ext().attn_sel_fwd(q, k, v, o, lse, scale, kblk, kpos, qoff)
        ctx.save_for_backward(q, k, v, o, lse, kblk, kpos, qoff)
        ctx.scale = scale
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, do, _dlse):
        from ._ext import ext
        q, k, v, o, lse, kblk, kpos, qoff = ctx.saved_tensors
        do = _kernel_ready(do.to(torch.bfloat16))
        D = torch.empty_like(lse)
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
        dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
        ext().attn_sel_bwd(q, k, v, o, lse, do, D, dq, dk, dv, ctx.scale, kblk, kpos, qoff)
        return dq.to(torch.bfloat16), dk.to(torch.bfloat16), dv.to(torch.bfloat16), None, None, None, None


def flash_attention_blocks(q, k, v, kblk, kpos, qoff, scale):
    """Query groups over selected 64-key blocks without gathering them.

    q [E, Lq, nh, hd] (E = B x groups), k / v [B, Lsrc, nh, hd]; entry e attends to the key
    blocks ``kblk[e]`` (int [E, nblk], block j = source rows [64 j, 64 j + 64) of batch
    e // (E // B)), whose keys sit at the absolute positions ``kpos`` [E, 64 nblk]; its queries
    start at position ``qoff[e]``.  Block indices are clamped to the source."""
    nb_max = k.shape[1] // 64 - 1
    kb = kblk.to(device=q.device, dtype=torch.int32).clamp(0, nb_max).contiguous()
    kp = kpos.to(device=q.device, dtype=torch.int32).contiguous()
    qo = qoff.to(device=q.device, dtype=torch.int32).contiguous()
    return _FlashAttnSel.apply(q, k, v, kb, kp, qo, float(scale))[0]


_ENABLED = [True]


class use_kernels:
    """``with use_kernels(False):`` runs the tensor-expression paths instead of the
    kernels (benchmarks and parity checks against the same module)."""

    def __init__(self, on: bool):
        self.on, self.prev = on, None

    def __enter__(self):
        self.prev, _ENABLED[0] = _ENABLED[0], self.on

    def __exit__(self, *exc):
        _ENABLED[0] = self.prev


def kernel_supported(q, k, v) -> bool:
    return (_ENABLED[0] and q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
            and q.shape[-1] in (64, 128))


def flash_attention_lse(q, k, v, scale, window=None, q_offset=0, kpos=None, qoff=None):
    """The kernels' forward with its base-2 row log-sum-exp: (o, lse [B, nh, Lq]).

    ``kpos`` (int32 [B, Lk]) gives every key an absolute position (compressed or gathered
    key blocks); ``qoff`` (int32 [B]) gives every batch entry its own query offset."""
    kp = None if kpos is None else kpos.to(device=q.device, dtype=torch.int32).contiguous()
    qo = None if qoff is None else qoff.to(device=q.device, dtype=torch.int32).contiguous()
    return _FlashAttn.apply(q, k, v, float(scale), int(window or 0), int(q_offset), kp, qo)


def attention_probsum(q, k, lse, scale, window=None, q_offset=0, kpos=None, qoff=None):
    """Head-summed softmax probabilities [B, Lq, Lk] (fp32) of a forward whose ``lse``
    is given -- the NSA block importance.  No gradient."""
    from ._ext import ext
    q, k = _kernel_ready(q.detach()), _kernel_ready(k.detach())
    imp = torch.empty(q.shape[0], q.shape[1], k.shape[1], dtype=torch.float32, device=q.device)
    kp = None if kpos is None else kpos.to(device=q.device, dtype=torch.int32).contiguous()
    qo = None if qoff is None else qoff.to(device=q.device, dtype=torch.int32).contiguous()
    ext().attn_probsum(q, k, lse, imp, float(scale), int(window or 0), int(q_offset), kp, qo)
    return imp


def flash_attention(q, k, v, scale=None, causal=True, window=None, q_offset=0, force_kernel=False,
                    kpos=None, qoff=None):
    """q (B, Lq, nh, hd), k/v (B, Lk, nh, hd) -> (B, Lq, nh, hd).

    Query i sits at absolute position ``q_offset + i`` (``qoff[b] + i`` when given) and
    sees keys at positions <= its own (within ``window`` tokens when given); key j sits
    at position j, or ``kpos[b, j]``."""
    hd = q.shape[-1]
    scale = scale if scale is not None else hd ** -0.5
    tables = kpos is not None or qoff is not None
    full = window is None and q_offset == 0 and q.shape[1] == k.shape[1] and not tables
    # Full causal attention stays on torch's fused attention, which dispatches to a
    # Blackwell-native library kernel (0.9-1.4 PFLOP/s forward on B200 against 0.15-0.2
    # for these mma.sync kernels); windows, decode offsets and position tables, which it
    # can only take as a dense mask, run the kernels here (7-16x the masked path).
    if (not full or force_kernel) and causal and kernel_supported(q, k, v):
        return flash_attention_lse(q, k, v, scale, window, q_offset, kpos, qoff)[0]
    if tables:
        raise ValueError("key-position / query-offset tables need bf16 CUDA inputs with head dim 64 or 128")
    if full:
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=causal, scale=scale)
        return o.transpose(1, 2)
    return _blocked(q, k, v, scale, window, q_offset)
