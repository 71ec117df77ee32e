"""Training step and loop (the public training API).

``Trainer`` builds the model from a preset / argparse namespace, re-homes its
parameters into the flat optimizer buffers, and runs steps:

* ``step_device(tokens, labels, book)`` -- one optimizer step on device tensors,
  returns the loss as a device scalar (no host sync);
* ``train_step(batch)`` -- the end-to-end call a user makes: copies the batch
  from (pinned) host memory, runs the step, returns the loss as a Python float.

Data parallelism: with ``world > 1`` the flat gradient is averaged over ranks
(NCCL all-reduce) before the update -- the reference's ``pmean`` over
``data``/``gpus`` (``training/train_helpers.py:2123-2196``) -- or, with
``sharded=True``, reduce-scattered so each rank updates only its shard of the
flat buffer and the updated parameters are all-gathered (ZeRO-1/2 style).
"""
from __future__ import annotations

import math
import time
from typing import Optional

import torch
import torch.distributed as dist

from ..encoding import get_tokenizer, set_token_mode
from ..models.registry import build_model, architecture_from_args, architecture_has_attention
from .optim import FlatAdam, cosine_schedule


class Trainer:
    def __init__(self, args, device: Optional[torch.device] = None, world: int = 1, rank: int = 0,
                 group=None, total_steps: int = 1000, seed: int = 0, sharded: bool = False):
        self.args = args
        self.device = device or torch.device("cuda" if torch.cuda.is_available() else "cpu")
        self.world, self.rank, self.group = world, rank, group
        set_token_mode(args.token_mode)
        self.tok = get_tokenizer(args.token_mode)
        torch.manual_seed(seed)
        self.model = build_model(args).to(self.device)
        arch = architecture_from_args(args)
        attn_only = arch in ("transformer", "nsa")
        if world > 1:
            # identical initial parameters on every rank (broadcast_one_to_all in the reference)
            for p in self.model.parameters():
                dist.broadcast(p.data, 0, group=group)
        lr_base = float(getattr(args, "ssm_lr_base", 1e-3))
        lr = lr_base * float(getattr(args, "lr_factor", 1.0))
        self.opt = FlatAdam(self.model, lr=lr, ssm_lr=lr_base,
                            weight_decay=float(getattr(args, "weight_decay", 0.05)),
                            max_grad_norm=float(getattr(args, "max_grad_norm", 1.0)),
                            opt_config=str(getattr(args, "opt_config", "standard")),
                            attention_model=attn_only)
        self.total_steps = total_steps
        self.warmup_steps = int(round(float(getattr(args, "warmup_end", 0.01)) * total_steps))
        lr_min = float(getattr(args, "lr_min", 0.0) or 0.0)
        self.lr_min_frac = (lr_min / lr) if lr_min > 0 else 0.05
        self.ignore_times = bool(getattr(args, "ignore_times", False))
        self.sharded = sharded and world > 1
        self.step_idx = 0
        self._sumsq_all = torch.zeros(1, device=self.device)

    # -- one step -------------------------------------------------------------------------
    def _reduce_grads(self):
        if self.world == 1:
            return None
        g = self.opt.grad
        if not self.sharded:
            g.div_(self.world)
            dist.all_reduce(g, group=self.group)
            return None
        raise NotImplementedError

    def step_device(self, tokens, labels, book=None):
        self.opt.zero_grad()
        loss, ce_pos = self.model.loss(tokens, book, labels, ignore_times=self.ignore_times,
                                       tokenizer=self.tok)
        loss.backward()
        self._reduce_grads()
        scale = cosine_schedule(self.step_idx + 1, self.warmup_steps, self.total_steps, self.lr_min_frac)
        self.opt.step(lr_scale=scale)
        self.step_idx += 1
        return loss.detach()

    def to_device(self, batch):
        return tuple(t.to(self.device, non_blocking=True) if t is not None else None for t in batch)

    def train_step(self, batch) -> float:
        """End-to-end step from host tensors ``(tokens, labels, book)``; returns the loss."""
        tokens, labels, book = self.to_device(batch)
        loss = self.step_device(tokens, labels, book)
        return float(loss.item())

    @torch.no_grad()
    def eval_loss(self, tokens, labels, book=None) -> float:
        loss, _ = self.model.loss(tokens.to(self.device), book.to(self.device) if book is not None else None,
                                  labels.to(self.device), ignore_times=self.ignore_times, tokenizer=self.tok)
        return float(loss)
