"""Normalisation epsilons of Mamba3 checkpoints trained before the epsilon fix.

Older reference checkpoints were trained with ``RMSNorm(N)`` / ``RMSNorm(d_inner)``
where the positional argument is Flax's *epsilon*: the B/C norms used
``eps = d_state`` and ``out_norm`` used ``eps = d_inner``, which nearly disables
them; weights learned under that regime need the same epsilons at inference
(``src/base_model/models/legacy_norm.py``).  Opt-in: ``MAMBA3_LEGACY_NORM=1``
in the environment (read by ``build_model``) or ``apply_legacy_norm(model)``.
Both the torch path and the CUDA kernels read the epsilons from the modules.
"""
from __future__ import annotations

import os

import torch.nn as nn


def legacy_norm_enabled() -> bool:
    return os.environ.get("MAMBA3_LEGACY_NORM", "").strip() not in ("", "0", "false", "False")


def apply_legacy_norm(model: nn.Module) -> int:
    """Set the legacy epsilons on every Mamba3 mixer; returns how many were changed."""
    from .mamba3 import Mamba3
    n = 0
    for m in model.modules():
        if isinstance(m, Mamba3):
            m.B_norm.eps = float(m.dims.d_state)
            m.C_norm.eps = float(m.dims.d_state)
            m.out_norm.eps = float(m.dims.d_inner)
            n += 1
    return n
