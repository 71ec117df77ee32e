"""BookDiT: a patch-token velocity model over chart horizons, conditioned on a context.

An alternative backbone to ``dit.FrameDiT`` (one token per frame): the horizon is cut
into patches of ``patch`` frames, the flow time and an MLP embedding of the last
``context`` observed frames condition every block through adaLN-zero modulation.
Training and sampling use the rectified-flow convention of ``flow.py`` (t = 0 data,
t = 1 noise, target eps - x0); ``bind_bookdit`` turns a model and its context into a
``flow.ModelFn`` so every post-training trainer of ``posttraining.py`` applies.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .flow import RectifiedFlow, fm_loss, interpolate, velocity_target
from .frames import resample_frames  # noqa: F401  (re-export)
from .representation import decode_frames, encode_frames  # noqa: F401  (re-export)


# ---------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------


def timestep_embedding(t: torch.Tensor, dim: int) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    a = t.float()[:, None] * 1000.0 * freqs[None]
    return torch.cat([torch.cos(a), torch.sin(a)], -1)


class DiTBlock(nn.Module):
    def __init__(self, d: int, heads: int):
        super().__init__()
        self.n1 = nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        self.attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.n2 = nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        self.mlp = nn.Sequential(nn.Linear(d, 4 * d), nn.GELU(approximate="tanh"), nn.Linear(4 * d, d))
        self.ada = nn.Linear(d, 6 * d)
        nn.init.zeros_(self.ada.weight)
        nn.init.zeros_(self.ada.bias)

    def forward(self, x, c):
        s1, b1, g1, s2, b2, g2 = self.ada(F.silu(c))[:, None].chunk(6, -1)
        h = self.n1(x) * (1 + s1) + b1
        x = x + g1 * self.attn(h, h, h, need_weights=False)[0]
        h = self.n2(x) * (1 + s2) + b2
        return x + g2 * self.mlp(h)


class BookDiT(nn.Module):
    """Velocity model v(x_t, t | context) over (B, T, C) chart horizons."""

    def __init__(self, channels: int, horizon: int, context: int, d: int = 128, depth: int = 4, heads: int = 4,
                 patch: int = 4):
        super().__init__()
        assert horizon % patch == 0
        self.C, self.T, self.p = channels, horizon, patch
        self.inp = nn.Linear(channels * patch, d)
        self.pos = nn.Parameter(torch.zeros(1, horizon // patch, d))
        self.ctx = nn.Sequential(nn.Linear(channels * context, d), nn.SiLU(), nn.Linear(d, d))
        self.temb = nn.Sequential(nn.Linear(d, d), nn.SiLU(), nn.Linear(d, d))
        self.blocks = nn.ModuleList([DiTBlock(d, heads) for _ in range(depth)])
        self.norm = nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        self.out = nn.Linear(d, channels * patch)
        nn.init.zeros_(self.out.weight)
        nn.init.zeros_(self.out.bias)
        self.d = d

    def forward(self, x, t, ctx):
        B = x.shape[0]
        h = self.inp(x.reshape(B, self.T // self.p, self.p * self.C)) + self.pos
        c = self.temb(timestep_embedding(t, self.d)) + self.ctx(ctx.reshape(B, -1))
        for blk in self.blocks:
            h = blk(h, c)
        return self.out(self.norm(h)).reshape(B, self.T, self.C)


def bind_bookdit(model: "BookDiT", ctx: torch.Tensor):
    """flow.ModelFn of a BookDiT for the context frames ``ctx`` (B, K, C)."""
    return lambda x_t, t: model(x_t, t, ctx)


def flow_matching_loss(model: "BookDiT", x0: torch.Tensor, ctx: torch.Tensor, weights=None, generator=None):
    """Rectified-flow loss on clean horizons x0 (B, T, C) given contexts (B, K, C)."""
    B = x0.shape[0]
    t = torch.rand(B, device=x0.device, generator=generator)
    eps = torch.randn(x0.shape, device=x0.device, generator=generator)
    return fm_loss(model(interpolate(x0, eps, t), t, ctx), velocity_target(x0, eps), weight=weights)


@torch.no_grad()
def sample(model: "BookDiT", ctx: torch.Tensor, steps: int = 16, generator=None) -> torch.Tensor:
    """Euler ODE sample of horizons for each context."""
    return RectifiedFlow(steps).sample_ode(bind_bookdit(model, ctx), (ctx.shape[0], model.T, model.C),
                                           ctx.device, generator=generator)
