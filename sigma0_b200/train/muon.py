"""Muon for the 2-D dense kernels (orthogonalised momentum), Adam/AdamW for the rest.

The reference's ``opt_config="muon"`` routes every 2-D ``kernel`` leaf through
``optax.contrib.scale_by_muon`` (Nesterov momentum, Newton-Schulz
orthogonalisation), then weight decay and the Muon learning rate; SSM leaves
use Adam and the rest AdamW (``training/train_helpers.py:645-700``).

``orthogonalize`` is the quintic Newton-Schulz iteration of Keller Jordan's
Muon (coefficients (3.4445, -4.7750, 2.0315), five steps, bf16-safe scaling by
the Frobenius norm), applied to the update matrix; the result is scaled by
``sqrt(max(1, rows/cols))`` so its RMS does not depend on the aspect ratio.
``FlatMuon`` keeps the flat-buffer layout of ``FlatAdam`` (one global-norm
clip over all gradients), runs the fused Adam kernel on the non-Muon slices
and Muon on each kernel slice.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .optim import FlatAdam

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def orthogonalize(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    a, b, c = NS_COEFFS
    X = G.to(torch.bfloat16 if G.is_cuda else torch.float32)
    transpose = X.shape[0] > X.shape[1]
    if transpose:
        X = X.T
    X = X / (X.norm() + eps)
    for _ in range(steps):
        A = X @ X.T
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transpose:
        X = X.T
    return X.to(G.dtype)


def is_muon_leaf(name: str, p: torch.Tensor) -> bool:
    return name.endswith("kernel") and p.dim() == 2 and "embedding" not in name


class FlatMuon(FlatAdam):
    def __init__(self, model, lr: float, ssm_lr: float, muon_lr: float = 0.02, muon_wd: Optional[float] = None,
                 momentum: float = 0.95, nesterov: bool = True, **kw):
        super().__init__(model, lr=lr, ssm_lr=ssm_lr, **kw)
        self.muon_lr = muon_lr
        self.muon_wd = kw.get("weight_decay", 0.05) if muon_wd is None else muon_wd
        self.mom, self.nesterov = momentum, nesterov
        named = dict(model.named_parameters())
        self.muon_names = [n for n in self.names if is_muon_leaf(n, named[n])]
        self._muon_buf = {n: torch.zeros_like(named[n]) for n in self.muon_names}
        self._named = named

    def step(self, lr_scale: float = 1.0, grad_sumsq: Optional[torch.Tensor] = None):
        if grad_sumsq is None:
            grad_sumsq = (self.grad * self.grad).sum().reshape(1)
        nrm = float(torch.sqrt(grad_sumsq))
        clip = 1.0 if (self.max_grad_norm <= 0 or nrm < self.max_grad_norm) else self.max_grad_norm / nrm
        # Muon slices: update here, then hide their gradients from the Adam pass
        lr = self.muon_lr * lr_scale
        with torch.no_grad():
            for n in self.muon_names:
                lo, hi = self.slices[n]
                p = self._named[n]
                g = self.grad[lo:hi].view_as(p) * clip
                buf = self._muon_buf[n]
                buf.mul_(self.mom).add_(g)
                upd = g.add(buf, alpha=self.mom) if self.nesterov else buf
                o = orthogonalize(upd) * math.sqrt(max(1.0, p.shape[0] / p.shape[1]))
                p.mul_(1 - lr * self.muon_wd).sub_(lr * o)
            saved = {}
            for n in self.muon_names:
                lo, hi = self.slices[n]
                saved[n] = (self.m[lo:hi].clone(), self.v[lo:hi].clone(), self.flat[lo:hi].clone())
        super().step(lr_scale=lr_scale, grad_sumsq=grad_sumsq)
        with torch.no_grad():   # the Adam pass must not touch Muon slices
            for n, (m, v, p) in saved.items():
                lo, hi = self.slices[n]
                self.m[lo:hi].copy_(m)
                self.v[lo:hi].copy_(v)
                self.flat[lo:hi].copy_(p)
            if self.shadow is not None:
                for n in self.muon_names:
                    lo, hi = self.slices[n]
                    self.shadow[lo:hi].copy_(self.flat[lo:hi])
