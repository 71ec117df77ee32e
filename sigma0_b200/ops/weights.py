"""bf16 compute copies of float32 master weights.

The fused optimizer writes a bf16 shadow of every parameter in the same pass
that updates the float32 master (``csrc/fused_ops.cu`` ``adam_k``); layers
fetch their GEMM operands here instead of casting every step.  Parameters
without a registered shadow are cast on the fly.
"""
from __future__ import annotations

from typing import Dict

import torch
import torch.nn.functional as F

_SHADOW: Dict[int, torch.Tensor] = {}
_PADDED: Dict[tuple, torch.Tensor] = {}


def register(param: torch.Tensor, shadow: torch.Tensor) -> None:
    _SHADOW[id(param)] = shadow


def clear() -> None:
    _SHADOW.clear()
    _PADDED.clear()


def freeze(module: torch.nn.Module) -> None:
    """Inference: cache a bf16 copy of every parameter once (and, lazily, the
    padded GEMM operands), so decode steps stop re-casting float32 weights."""
    for p in module.parameters():
        if id(p) not in _SHADOW:
            _SHADOW[id(p)] = p.detach().to(torch.bfloat16)
            _PADDED[("frozen", id(p))] = _SHADOW[id(p)]


def bf16(param: torch.Tensor) -> torch.Tensor:
    s = _SHADOW.get(id(param))
    if s is not None and s.data_ptr() != 0:
        return s
    return param.detach().to(torch.bfloat16)


def bf16_padded(param: torch.Tensor, cols: int) -> torch.Tensor:
    """bf16 copy of a (rows, c) kernel zero-padded to ``cols`` columns."""
    w = bf16(param)
    if w.shape[1] == cols:
        return w
    frozen = ("frozen", id(param)) in _PADDED
    key = (id(param), cols)
    if frozen and key in _PADDED:
        return _PADDED[key]
    out = F.pad(w, (0, cols - w.shape[1]))
    if frozen:
        _PADDED[key] = out
    return out
