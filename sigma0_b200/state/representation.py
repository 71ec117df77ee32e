"""Chart coordinates for book frames: any real-valued chart decodes to a valid book.

Per level k (level-major, 4 channels), following the channel definition of the
reference's ``state/representation.py:53-130`` so charts, normalisers and
checkpoints carry over:

    k = 0:  log(ask_1 - bid_1)   ask_size_1   mid_t - mid_{t-1} (0 at t=0)   bid_size_1
    k > 0:  log(ask_k+1 - ask_k) ask_size     log(bid_k - bid_k+1)           bid_size
    [4L]:   log1p(events folded into the frame)     (optional activity channel)

Decoding takes exp of the spread and gap channels and rebuilds the ladders with
cumulative sums from the mid (anchored at the first frame's mid), so the spread
is positive and the ladders strictly monotone by construction.  ``min_gap`` floors
the log arguments in price units (1 for integer LOBSTER prices).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch


def chart_channels(levels: int, with_activity: bool = False) -> int:
    return 4 * levels + int(with_activity)


def encode_frames(book: np.ndarray, events_per_frame: Optional[np.ndarray] = None,
                  min_gap: float = 1.0) -> Tuple[np.ndarray, float]:
    """(T, 4L) raw frames -> (chart (T, 4L[+1]) float32, first-frame mid)."""
    f = np.asarray(book, dtype=np.float64)
    if f.ndim != 2 or f.shape[1] % 4:
        raise ValueError(f"expected (T, 4*levels) frames, got {f.shape}")
    ask, bid = f[:, 0::4], f[:, 2::4]
    mid = 0.5 * (ask[:, 0] + bid[:, 0])
    c = f.copy()
    c[:, 0] = np.log(np.maximum(ask[:, 0] - bid[:, 0], min_gap))
    c[:, 2] = np.concatenate([[0.0], np.diff(mid)])
    c[:, 4::4] = np.log(np.maximum(np.diff(ask, axis=1), min_gap))
    c[:, 6::4] = np.log(np.maximum(-np.diff(bid, axis=1), min_gap))
    if events_per_frame is not None:
        c = np.concatenate([c, np.log1p(np.asarray(events_per_frame, dtype=np.float64))[:, None]], 1)
    return c.astype(np.float32), float(mid[0])


def decode_frames(chart: np.ndarray, anchor_mid: float) -> np.ndarray:
    """Exact inverse of :func:`encode_frames` (the activity channel is dropped)."""
    c = np.asarray(chart, dtype=np.float64)
    nb = c.shape[1] // 4 * 4
    out = c[:, :nb].copy()
    mid = anchor_mid + np.cumsum(c[:, 2])
    half = 0.5 * np.exp(c[:, 0])
    out[:, 0::4] = (mid + half)[:, None] + np.concatenate(
        [np.zeros((len(c), 1)), np.cumsum(np.exp(c[:, 4:nb:4]), 1)], 1)
    out[:, 2::4] = (mid - half)[:, None] - np.concatenate(
        [np.zeros((len(c), 1)), np.cumsum(np.exp(c[:, 6:nb:4]), 1)], 1)
    return out.astype(np.float32)


def decode_frames_torch(chart: torch.Tensor, anchor_mid: torch.Tensor) -> torch.Tensor:
    """Differentiable batched decode: (B, T, 4L[+1]) and (B,) anchors -> (B, T, 4L)."""
    if chart.dim() != 3:
        raise ValueError(f"expected (B, T, C), got {tuple(chart.shape)}")
    nb = chart.shape[-1] // 4 * 4
    c = chart[..., :nb]
    mid = anchor_mid.reshape(-1, 1).to(c.dtype) + torch.cumsum(c[..., 2], 1)
    half = 0.5 * torch.exp(c[..., 0])
    zero = torch.zeros_like(mid)[..., None]
    ask = (mid + half)[..., None] + torch.cat([zero, torch.cumsum(torch.exp(c[..., 4::4]), -1)], -1)
    bid = (mid - half)[..., None] - torch.cat([zero, torch.cumsum(torch.exp(c[..., 6::4]), -1)], -1)
    out = torch.stack([ask, c[..., 1::4], bid, c[..., 3::4]], -1)       # (B, T, L, 4)
    return out.flatten(-2)


class ChartNormalizer:
    """One mean and std per channel over the training split (shipped in checkpoints)."""

    def __init__(self, mean, std, std_floor: float = 1e-6):
        self.mean = np.asarray(mean, dtype=np.float32)
        self.std = np.maximum(np.asarray(std, dtype=np.float32), std_floor)

    @classmethod
    def fit(cls, chart: np.ndarray) -> "ChartNormalizer":
        c = np.asarray(chart, dtype=np.float64)
        return cls(c.mean(0), c.std(0))

    def normalize(self, chart):
        return ((np.asarray(chart) - self.mean) / self.std).astype(np.float32)

    def denormalize(self, chart):
        return (np.asarray(chart) * self.std + self.mean).astype(np.float32)

    def denormalize_torch(self, chart: torch.Tensor) -> torch.Tensor:
        return chart * torch.as_tensor(self.std, device=chart.device, dtype=chart.dtype) + \
            torch.as_tensor(self.mean, device=chart.device, dtype=chart.dtype)

    def state_dict(self) -> dict:
        return {"mean": self.mean.tolist(), "std": self.std.tolist()}

    @classmethod
    def from_state_dict(cls, d: dict) -> "ChartNormalizer":
        return cls(d["mean"], d["std"])
