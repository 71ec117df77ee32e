"""FrameDiT: a diffusion transformer over book frames, one token per frame.

Architecture (the reference's ``state/dit.py:165-235``; the parameter tree --
module names and shapes -- is the same so state dicts load either way):

* input projection of ``cat([x_t, cond, mask])`` (``2C + 1`` columns; ``C`` when
  unconditional).  The conditioning columns start at zero, so a model
  initialised from an unconditional checkpoint behaves identically at step 0;
* flow time: sinusoid of ``1000 t`` (cos first, fp32) -> MLP -> a shared 6-way
  projection; every block adds its own learned 6 x H table (shift/scale/gate for
  attention and MLP: the Wan-style AdaLN);
* blocks: LayerNorm (no affine) -> bidirectional attention with per-head RMSNorm on
  q and k and interleaved RoPE from an fp32 cache sized ``max_seq_len`` -> gated
  residual; the same around a GELU(tanh) MLP;
* final LayerNorm and a zero-initialised velocity head (the model starts at v = 0).

``bind_condition(model, context, obs_mask)`` closes the model over clean context
frames (``obs_mask`` 1 = given) and returns a ``flow.ModelFn``; the mask channel the
model sees is the complement (1 = generate).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class FrameDiTConfig:
    channels: int = 41
    hidden: int = 128
    depth: int = 4
    heads: int = 4
    mlp_ratio: float = 4.0
    max_seq_len: int = 4096
    freq_dim: int = 256
    conditional: bool = True

    @property
    def head_dim(self) -> int:
        if self.hidden % self.heads:
            raise ValueError("hidden must be divisible by heads")
        return self.hidden // self.heads

    @property
    def input_dim(self) -> int:
        return 2 * self.channels + 1 if self.conditional else self.channels


def timestep_embedding(t: torch.Tensor, dim: int) -> torch.Tensor:
    half = dim // 2
    k = torch.arange(half, device=t.device, dtype=torch.float32)
    ang = (1000.0 * t.float())[:, None] * torch.exp(k * (-math.log(10000.0) / half))[None]
    return torch.cat([ang.cos(), ang.sin()], -1).to(t.dtype)


class RotaryEmbedding(nn.Module):
    """Interleaved-pair RoPE; cos/sin tables in fp32, built once for max_seq_len."""

    def __init__(self, head_dim: int, max_seq_len: int, base: float = 10000.0):
        super().__init__()
        if head_dim % 2:
            raise ValueError("RoPE needs an even head_dim")
        inv = base ** (-torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
        ang = torch.arange(max_seq_len, dtype=torch.float32)[:, None] * inv[None]
        self.register_buffer("cos", ang.cos(), persistent=False)
        self.register_buffer("sin", ang.sin(), persistent=False)
        self.max_seq_len = max_seq_len

    def rotate(self, x: torch.Tensor) -> torch.Tensor:
        L = x.shape[-2]
        if L > self.max_seq_len:
            raise ValueError(f"sequence of {L} frames exceeds the RoPE table ({self.max_seq_len})")
        c, s = self.cos[:L].float(), self.sin[:L].float()
        xf = x.float().unflatten(-1, (-1, 2))
        a, b = xf[..., 0], xf[..., 1]
        return torch.stack([a * c - b * s, a * s + b * c], -1).flatten(-2).to(x.dtype)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


class _Attention(nn.Module):
    def __init__(self, cfg: FrameDiTConfig, rope: RotaryEmbedding):
        super().__init__()
        H = cfg.hidden
        self.q, self.k, self.v, self.o = (nn.Linear(H, H) for _ in range(4))
        self.q_norm, self.k_norm = RMSNorm(cfg.head_dim), RMSNorm(cfg.head_dim)
        self.heads = cfg.heads
        self.rope = rope

    def forward(self, x):
        B, L, H = x.shape
        split = lambda y: y.view(B, L, self.heads, H // self.heads).transpose(1, 2)
        q = self.rope.rotate(self.q_norm(split(self.q(x))))
        k = self.rope.rotate(self.k_norm(split(self.k(x))))
        y = F.scaled_dot_product_attention(q, k, split(self.v(x)))
        return self.o(y.transpose(1, 2).reshape(B, L, H))


class _WanBlock(nn.Module):
    def __init__(self, cfg: FrameDiTConfig, rope: RotaryEmbedding):
        super().__init__()
        H = cfg.hidden
        self.norm1 = nn.LayerNorm(H, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(H, elementwise_affine=False)
        self.attn = _Attention(cfg, rope)
        F_ = int(H * cfg.mlp_ratio)
        self.ffn = nn.Sequential(nn.Linear(H, F_), nn.GELU(approximate="tanh"), nn.Linear(F_, H))
        self.modulation = nn.Parameter(torch.randn(1, 6, H) / math.sqrt(H))

    def forward(self, x, e):
        sh1, sc1, g1, sh2, sc2, g2 = (self.modulation + e).unbind(1)
        x = x + g1[:, None] * self.attn(self.norm1(x) * (1 + sc1[:, None]) + sh1[:, None])
        return x + g2[:, None] * self.ffn(self.norm2(x) * (1 + sc2[:, None]) + sh2[:, None])


class FrameDiT(nn.Module):
    """forward(x (B, L, input_dim), t (B,)) -> velocity (B, L, channels)."""

    def __init__(self, cfg: FrameDiTConfig):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden
        self.input_proj = nn.Linear(cfg.input_dim, H)
        self.time_embedding = nn.Sequential(nn.Linear(cfg.freq_dim, H), nn.SiLU(), nn.Linear(H, H))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(H, 6 * H))
        rope = RotaryEmbedding(cfg.head_dim, cfg.max_seq_len)
        self.blocks = nn.ModuleList([_WanBlock(cfg, rope) for _ in range(cfg.depth)])
        self.final_norm = nn.LayerNorm(H)
        self.velocity_head = nn.Linear(H, cfg.channels)
        with torch.no_grad():
            self.velocity_head.weight.zero_()
            self.velocity_head.bias.zero_()
            if cfg.conditional:
                self.input_proj.weight[:, cfg.channels:].zero_()

    def forward(self, x, t):
        h = self.input_proj(x)
        e = self.time_projection(self.time_embedding(timestep_embedding(t, self.cfg.freq_dim)))
        e = e.view(-1, 6, self.cfg.hidden)
        for blk in self.blocks:
            h = blk(h, e)
        return self.velocity_head(self.final_norm(h))


def bind_condition(model: FrameDiT, context: torch.Tensor, obs_mask: torch.Tensor):
    """ModelFn of a conditional FrameDiT given clean ``context`` (B, L, C) where
    ``obs_mask`` (B, L) is 1."""
    if not model.cfg.conditional:
        raise ValueError("the model was built unconditional")
    obs = obs_mask.to(context.dtype)[..., None]
    cond, gen = context * obs, 1.0 - obs

    def fn(x_t, t):
        return model(torch.cat([x_t, cond, gen], -1), t)

    return fn


def bind_unconditional(model: FrameDiT):
    """ModelFn with nothing given (every frame generated)."""
    if not model.cfg.conditional:
        return model

    def fn(x_t, t):
        zeros = torch.zeros_like(x_t)
        ones = torch.ones_like(x_t[..., :1])
        return model(torch.cat([x_t, zeros, ones], -1), t)

    return fn
