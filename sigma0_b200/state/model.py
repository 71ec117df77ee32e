"""Book-state world model: wall-clock frames, a chart representation, a DiT and flow matching.

The reference's ``state`` package (PyTorch) models the order book like video:
frames on a uniform wall clock (``frames.py``: forward-filled book state at
every ``interval_ns``), a relative "chart" representation (``representation.py``:
log spread, mid changes, log level gaps, log sizes), a diffusion transformer
(``dit.py``, WanDiT) trained with rectified flow matching (``flow.py``), rewards
and post-training trainers (``rewards.py``, ``posttraining/``).  This module
implements the same pipeline:

* ``resample_frames`` -- forward-fill book rows onto a ``interval_ns`` grid and
  count the events folded into each frame;
* ``encode_chart`` / ``decode_chart`` -- (T, 4L) raw frames <-> chart channels
  (first-frame mid as the anchor; exact inverse);
* ``BookDiT`` -- patchify the horizon into tokens, transformer blocks with
  adaLN modulation by the flow time and a context embedding (the last observed
  frames), predict the velocity;
* ``flow_matching_loss`` / ``sample`` -- rectified flow: x_t = (1-t) x0 + t x1,
  target v = x1 - x0; Euler integration from noise;
* ``reward_weighted_loss`` -- advantage-weighted flow matching (the
  reward-weighted post-training family: frames from the model are re-weighted
  by ``exp(A / beta)`` of a reward), with ``spread_reward`` and
  ``smoothness_reward`` as example rewards.
"""
from __future__ import annotations

import math
from typing import Callable, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

# ---------------------------------------------------------------------------
# frames and chart
# ---------------------------------------------------------------------------


def resample_frames(books: np.ndarray, interval_ns: int = 1_000_000, n_frames: Optional[int] = None):
    """Book rows ``[dmid, time_s, time_ns, L2...]`` -> (frames (T, 4L), events_per_frame (T,)).

    frame[k] = the state of the last event with time <= grid[k] (forward fill)."""
    b = np.asarray(books)
    t = b[:, 1].astype(np.int64) * 1_000_000_000 + b[:, 2].astype(np.int64)
    grid0 = t[0]
    T = n_frames or int((t[-1] - grid0) // interval_ns) + 1
    grid = grid0 + np.arange(T, dtype=np.int64) * interval_ns
    idx = np.searchsorted(t, grid, side="right") - 1
    idx = np.clip(idx, 0, len(t) - 1)
    counts = np.diff(np.concatenate([[0], np.searchsorted(t, grid, side="right")]))
    return b[idx, 3:].astype(np.float64), counts


def encode_chart(frames: np.ndarray, min_gap: float = 1.0) -> Tuple[np.ndarray, float]:
    """(T, 4L) raw frames -> chart (T, 4L) and the first-frame mid (anchor).

    Channels per level k: ask gap (log; level 0: log spread), log ask size,
    bid gap (log; level 0: mid change), log bid size."""
    f = np.asarray(frames, dtype=np.float64)
    L = f.shape[1] // 4
    ask, bid = f[:, 0::4], f[:, 2::4]
    mid = 0.5 * (ask[:, 0] + bid[:, 0])
    c = np.empty_like(f)
    c[:, 0] = np.log(np.maximum(ask[:, 0] - bid[:, 0], min_gap))
    c[:, 2] = np.concatenate([[0.0], np.diff(mid)])
    for k in range(1, L):
        c[:, 4 * k] = np.log(np.maximum(ask[:, k] - ask[:, k - 1], min_gap))
        c[:, 4 * k + 2] = np.log(np.maximum(bid[:, k - 1] - bid[:, k], min_gap))
    c[:, 1::4] = np.log1p(np.maximum(f[:, 1::4], 0))
    c[:, 3::4] = np.log1p(np.maximum(f[:, 3::4], 0))
    return c, float(mid[0])


def decode_chart(chart: np.ndarray, anchor: float) -> np.ndarray:
    c = np.asarray(chart, dtype=np.float64)
    L = c.shape[1] // 4
    mid = anchor + np.cumsum(c[:, 2])
    spread = np.exp(c[:, 0])
    f = np.empty_like(c)
    f[:, 0] = mid + spread / 2
    f[:, 2] = mid - spread / 2
    for k in range(1, L):
        f[:, 4 * k] = f[:, 4 * (k - 1)] + np.exp(c[:, 4 * k])
        f[:, 4 * k + 2] = f[:, 4 * (k - 1) + 2] - np.exp(c[:, 4 * k + 2])
    f[:, 1::4] = np.expm1(c[:, 1::4])
    f[:, 3::4] = np.expm1(c[:, 3::4])
    return f


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


def flow_matching_loss(model: BookDiT, x1: torch.Tensor, ctx: torch.Tensor, weights: Optional[torch.Tensor] = None):
    """Rectified flow: x_t = (1 - t) x0 + t x1 with x0 ~ N(0, I), regress v = x1 - x0."""
    B = x1.shape[0]
    t = torch.rand(B, device=x1.device)
    x0 = torch.randn_like(x1)
    xt = (1 - t)[:, None, None] * x0 + t[:, None, None] * x1
    err = ((model(xt, t, ctx) - (x1 - x0)) ** 2).mean((1, 2))
    if weights is not None:
        return (err * weights).sum() / weights.sum().clamp(min=1e-12)
    return err.mean()


@torch.no_grad()
def sample(model: BookDiT, ctx: torch.Tensor, steps: int = 16, generator=None) -> torch.Tensor:
    B = ctx.shape[0]
    x = torch.randn(B, model.T, model.C, device=ctx.device, generator=generator)
    for i in range(steps):
        t = torch.full((B,), i / steps, device=ctx.device)
        x = x + model(x, t, ctx) / steps
    return x


# ---------------------------------------------------------------------------
# rewards and reward-weighted post-training
# ---------------------------------------------------------------------------


def spread_reward(chart: torch.Tensor, target_log_spread: float) -> torch.Tensor:
    """Closeness of the level-0 log spread to a target, per sample."""
    return -((chart[..., 0] - target_log_spread) ** 2).mean(-1)


def smoothness_reward(chart: torch.Tensor) -> torch.Tensor:
    """Penalise frame-to-frame jumps of the mid (channel 2)."""
    return -(chart[..., 2] ** 2).mean(-1)


def reward_weighted_loss(model: BookDiT, ctx: torch.Tensor, reward: Callable[[torch.Tensor], torch.Tensor],
                         n_samples: int = 4, beta: float = 1.0, steps: int = 8):
    """Sample ``n_samples`` horizons per context, score them, and fit the model to its own
    samples weighted by ``softmax(A / beta)`` within each context (advantage-weighted
    flow matching)."""
    B = ctx.shape[0]
    rep = ctx.repeat_interleave(n_samples, 0)
    x = sample(model, rep, steps=steps)
    r = reward(x).reshape(B, n_samples)
    adv = r - r.mean(1, keepdim=True)
    w = torch.softmax(adv / beta, 1).reshape(-1) * n_samples
    return flow_matching_loss(model, x.detach(), rep, weights=w.detach()), r.mean()
