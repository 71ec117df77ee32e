"""Local steps with periodic outer synchronisation (DiLoCo / FedAvg).

Each rank runs ``inner_steps`` ordinary optimizer steps on its own data with no
gradient communication; then the ranks average their parameter change (the
pseudo-gradient ``global - local``) with one all-reduce of the flat parameter
buffer and apply an outer optimizer to the shared copy: Nesterov momentum SGD
for DiLoCo, plain averaging (outer lr 1, no momentum) for FedAvg.  The
reference runs the same scheme under ``shard_map`` (``training/train_helpers.py:2209-2320``,
``DiLoCoState`` ``:318``; CLI guards ``runtime/train.py:336-343``).

Works on any ``Trainer`` built with ``world=1`` (its own steps must not sync);
the process group is only used here.  The flat fp32 buffer makes the outer
step three vector ops and a single collective.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class DiLoCo:
    def __init__(self, trainer, inner_steps: int = 50, outer_lr: float = 0.7, outer_momentum: float = 0.9,
                 nesterov: bool = True, group=None, mode: str = "diloco"):
        if trainer.world != 1:
            raise ValueError("build the inner Trainer with world=1: DiLoCo does its own (outer) communication")
        if mode not in ("diloco", "fedavg"):
            raise ValueError(f"mode must be diloco or fedavg, not {mode!r}")
        self.tr, self.H, self.group = trainer, int(inner_steps), group
        self.mode = mode
        self.lr = 1.0 if mode == "fedavg" else outer_lr
        self.mu = 0.0 if mode == "fedavg" else outer_momentum
        self.nesterov = nesterov and mode == "diloco"
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        flat = trainer.opt.flat
        self.global_params = flat.detach().clone()
        if self.world > 1:      # start from identical parameters
            dist.broadcast(self.global_params, 0, group=group)
            flat.copy_(self.global_params)
            trainer.opt.refresh_shadow()
        self.momentum = torch.zeros_like(flat)
        self.inner = 0
        self.outer_steps = 0

    def step(self, tokens, labels, book=None):
        loss = self.tr.step_device(tokens, labels, book)
        self.inner += 1
        if self.inner % self.H == 0:
            self.outer_step()
        return loss

    @torch.no_grad()
    def outer_step(self):
        flat = self.tr.opt.flat
        delta = self.global_params - flat               # pseudo-gradient
        if self.world > 1:
            dist.all_reduce(delta, group=self.group)
            delta.div_(self.world)
        if self.mu > 0:
            self.momentum.mul_(self.mu).add_(delta)
            upd = delta + self.mu * self.momentum if self.nesterov else self.momentum
        else:
            upd = delta
        self.global_params.sub_(self.lr * upd)
        flat.copy_(self.global_params)
        self.tr.opt.refresh_shadow()
        self.outer_steps += 1
