"""Rotary and sinusoidal position encodings for the attention backbones.

``rotary_embedding``/``apply_rope`` follow the rotate-half convention of the
reference (``src/base_model/models/rope.py:24-120``): frequencies
``base^(-i/(d/2))``, the first half of the head dims paired with the second.
``sinusoidal`` matches the transformer's additive encoding
(``src/base_model/models/transformer.py:88-110``).
"""
from __future__ import annotations

import torch


def rotary_embedding(dim: int, seq_len: int, base: float = 10000.0, device=None, offset: int = 0):
    if dim % 2:
        raise ValueError(f"RoPE requires even dim, got {dim}")
    half = dim // 2
    inv = 1.0 / (base ** (torch.arange(half, dtype=torch.float32, device=device) / half))
    pos = torch.arange(offset, offset + seq_len, dtype=torch.float32, device=device)
    ang = torch.outer(pos, inv)
    return torch.cos(ang), torch.sin(ang)


def rope_at(dim: int, positions: torch.Tensor, base: float = 10000.0):
    half = dim // 2
    inv = 1.0 / (base ** (torch.arange(half, dtype=torch.float32, device=positions.device) / half))
    ang = positions.float()[..., None] * inv
    return torch.cos(ang), torch.sin(ang)


def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """q, k (..., L, nh, hd); cos/sin (L, hd/2) or broadcastable (..., L, 1, hd/2)."""
    if cos.dim() == 2:
        cos, sin = cos[:, None, :], sin[:, None, :]

    def rot(x):
        xf = x.float()
        h = xf.shape[-1] // 2
        x1, x2 = xf[..., :h], xf[..., h:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)
    return rot(q), rot(k)


def sinusoidal(L: int, d: int, device=None, offset: int = 0) -> torch.Tensor:
    pos = torch.arange(offset, offset + L, dtype=torch.float32, device=device)[:, None]
    dims = torch.arange(d, device=device)[None, :]
    ang = pos / torch.pow(10000.0, (2 * (dims // 2)).float() / d)
    return torch.where(dims % 2 == 0, torch.sin(ang), torch.cos(ang))


def sinusoidal_at(positions: torch.Tensor, d: int) -> torch.Tensor:
    pos = positions.float()[..., None]
    dims = torch.arange(d, device=positions.device)
    ang = pos / torch.pow(10000.0, (2 * (dims // 2)).float() / d)
    return torch.where(dims % 2 == 0, torch.sin(ang), torch.cos(ang))
