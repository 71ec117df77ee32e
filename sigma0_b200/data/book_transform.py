"""L2 book -> fixed volume image (the model's book input).

Same transform as the reference's ``transform_L2_state_numpy``
(``src/base_model/data/preproc.py:119-167``): prices are re-indexed relative to
the ceil-rounded mid into ``price_levels`` slots (slot ``price_levels//2`` is the
mid), ask volumes are negated, everything is divided by 1000, and the three
leading columns ``[delta_mid, time_s, time_ns]`` are normalised to fraction of
the trading day and fraction of a second.  Output width is ``3 + price_levels``
(503 for the production depth of 500).

``transform_books_torch`` is the batched device version used in the training
step; the numpy one is the oracle.
"""
from __future__ import annotations

import numpy as np
import torch


def transform_l2_numpy(book: np.ndarray, price_levels: int = 500, tick: int = 100) -> np.ndarray:
    """One book row ``[dmid, t_s, t_ns, ap1, av1, bp1, bv1, ...]`` -> (3 + price_levels,)."""
    head = np.asarray(book[:3], dtype=np.float32).copy()
    lv = np.asarray(book[3:], dtype=np.int64).reshape(-1, 2).copy()
    mid = int(np.ceil((lv[0, 0] + lv[1, 0]) / (2 * tick)) * tick)
    lv[:, 0] = (lv[:, 0] - mid) // tick + price_levels // 2
    keep = (lv[:, 0] >= 0) & (lv[:, 0] < 500)   # the reference hard-codes 500 here
    img = np.zeros(price_levels, dtype=np.int64)
    img[lv[keep, 0]] = lv[keep, 1]
    head[1] = (head[1] - 34200) / 23400
    head[2] = head[2] / 1e9
    img[price_levels // 2:] *= -1
    return np.concatenate([head, img.astype(np.float32) / 1000]).astype(np.float32)


def transform_books_numpy(books: np.ndarray, price_levels: int = 500, tick: int = 100) -> np.ndarray:
    return np.stack([transform_l2_numpy(b, price_levels, tick) for b in books])


def transform_books_torch(books: torch.Tensor, price_levels: int = 500, tick: int = 100) -> torch.Tensor:
    """(..., 3 + 4L) float64/int64 rows -> (..., 3 + price_levels) float32, vectorised."""
    shp = books.shape[:-1]
    b = books.reshape(-1, books.shape[-1])
    head = b[:, :3].to(torch.float64)
    lv = b[:, 3:].to(torch.int64).reshape(b.shape[0], -1, 2)
    mid = torch.ceil((lv[:, 0, 0] + lv[:, 1, 0]).to(torch.float64) / (2 * tick)).to(torch.int64) * tick
    idx = torch.div(lv[:, :, 0] - mid[:, None], tick, rounding_mode="floor") + price_levels // 2
    keep = (idx >= 0) & (idx < 500)
    img = torch.zeros(b.shape[0], price_levels, dtype=torch.int64, device=b.device)
    vals = torch.where(keep, lv[:, :, 1], torch.zeros_like(lv[:, :, 1]))
    safe = torch.where(keep, idx, torch.zeros_like(idx))
    # later levels overwrite earlier ones at equal slots, like numpy fancy assignment
    for j in range(idx.shape[1]):
        rows = torch.nonzero(keep[:, j], as_tuple=True)[0]
        img[rows, safe[rows, j]] = vals[rows, j]
    out_head = torch.stack([head[:, 0], (head[:, 1] - 34200) / 23400, head[:, 2] / 1e9], dim=1)
    img[:, price_levels // 2:] *= -1
    out = torch.cat([out_head.to(torch.float32), img.to(torch.float32) / 1000], dim=1)
    return out.reshape(*shp, 3 + price_levels)
