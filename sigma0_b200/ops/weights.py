"""bf16 compute copies of float32 master weights.

The fused optimizer writes a bf16 shadow of every parameter in the same pass
that updates the float32 master (``csrc/fused_ops.cu`` ``adam_k``); layers
fetch their GEMM operands here instead of casting every step.  Parameters
without a registered shadow are cast on the fly.

The shadow is stored on the parameter object itself, so its lifetime is the
parameter's (a registry keyed by ``id()`` would hand a dead parameter's shadow
to a new one that reuses the address).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def register(param: torch.Tensor, shadow: torch.Tensor) -> None:
    param._s0_shadow = shadow
    param._s0_padded = None


def clear(module: torch.nn.Module) -> None:
    for p in module.parameters():
        p._s0_shadow = None
        p._s0_padded = None


def freeze(module: torch.nn.Module) -> None:
    """Inference: cache a bf16 copy of every parameter once (and, lazily, the
    padded GEMM operands), so decode steps stop re-casting float32 weights.
    Call again (or ``clear``) after the float32 weights change."""
    for p in module.parameters():
        if getattr(p, "_s0_shadow", None) is None:
            p._s0_shadow = p.detach().to(torch.bfloat16)
        p._s0_padded = {}


def bf16(param: torch.Tensor) -> torch.Tensor:
    s = getattr(param, "_s0_shadow", None)
    if s is not None:
        return s
    return param.detach().to(torch.bfloat16)


def bf16_padded(param: torch.Tensor, cols: int) -> torch.Tensor:
    """bf16 copy of a (rows, c) kernel zero-padded to ``cols`` columns."""
    w = bf16(param)
    if w.shape[1] == cols:
        return w
    cache = getattr(param, "_s0_padded", None)   # a dict only for frozen (inference) weights
    if cache is not None and cols in cache:
        return cache[cols]
    out = F.pad(w, (0, cols - w.shape[1]))
    if cache is not None:
        cache[cols] = out
    return out
