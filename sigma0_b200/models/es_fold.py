"""Low-rank evolution-strategies perturbation of the dense projections (EGGROLL fold).

An ES population member evaluates the model with every selected projection
``x @ W`` replaced by ``x @ W + x @ A @ B^T``, where the factors ``A (in, r)`` and
``B (out, r)`` are sampled once per ES step (antithetic sign folded into ``A``);
``sigma = 0`` gives ``A = 0`` and an exactly unchanged forward
(``src/base_model/models/es_fold.py``).

``sample_factors`` draws the factors for the ``Dense`` modules whose qualified
names match ``include``; ``es_perturbation`` applies them with forward hooks for
the duration of a ``with`` block (no model code changes, and nothing is left
behind when the block exits); ``fold_kernel`` is the functional form.
"""
from __future__ import annotations

import contextlib
import math
import re
from typing import Dict, Optional

import torch
import torch.nn as nn

from .common import Dense


def fold_kernel(es: Optional[Dict], name: str, x: torch.Tensor, base: torch.Tensor) -> torch.Tensor:
    """``base + x @ A @ B^T`` if ``es[name]`` holds factors ``{"A", "B"}``, else ``base``."""
    if es is None or name not in es:
        return base
    ab = es[name]
    return base + (x.to(ab["A"].dtype) @ ab["A"]) @ ab["B"].T


def sample_factors(model: nn.Module, rank: int, sigma: float, seed: int, antithetic_sign: int = 1,
                   include: str = r".*(in_proj|out_proj|out2|decoder).*") -> Dict[str, Dict[str, torch.Tensor]]:
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, mod in model.named_modules():
        if isinstance(mod, Dense) and re.match(include, name):
            dev = mod.kernel.device
            A = torch.randn(mod.d_in, rank, generator=g) * (sigma / math.sqrt(rank)) * antithetic_sign
            B = torch.randn(mod.d_out, rank, generator=g)
            out[name] = {"A": A.to(dev), "B": B.to(dev)}
    return out


@contextlib.contextmanager
def es_perturbation(model: nn.Module, factors: Dict[str, Dict[str, torch.Tensor]]):
    """Apply the low-rank perturbation to matching ``Dense`` modules inside the block."""
    handles = []
    mods = dict(model.named_modules())
    for name, ab in factors.items():
        mod = mods[name]

        def hook(m, inputs, output, ab=ab):
            x = inputs[0]
            return output + ((x.to(ab["A"].dtype) @ ab["A"]) @ ab["B"].T).to(output.dtype)
        handles.append(mod.register_forward_hook(hook))
    try:
        yield
    finally:
        for h in handles:
            h.remove()
