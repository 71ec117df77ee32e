"""Flat-buffer optimizer: global-norm clip + grouped Adam/AdamW in one fused kernel per group.

Parameter routing follows the reference's ``standard`` configuration
(``training/train_helpers.py:534-568``): leaves named ``B``, ``Lambda_re``,
``Lambda_im``, ``log_step``, ``norm``, ``B_bias``, ``C_bias``, ``dt_bias`` or
``D`` go to the ``ssm`` group (Adam, ``ssm_lr``, no weight decay); every other
leaf goes to ``regular`` (AdamW, ``lr``, ``weight_decay``).  ``noBCdecay``,
``BandCdecay`` and ``BfastandCdecay`` change the leaf sets the same way the
reference does.  The whole update is preceded by ``clip_by_global_norm``
(``MAX_GRAD_NORM``, default 1.0).  Adam hyper-parameters are optax's
defaults (b1 0.9, b2 0.999, eps 1e-8, decoupled weight decay ``lr * wd * p``).

All parameters live in one float32 buffer (ssm group first), gradients in a
second; each ``nn.Parameter`` becomes a view, so autograd accumulates straight
into the flat gradient and the update is one kernel launch per group.  The same
kernel writes the bf16 compute copy used by the GEMMs.  On CPU the identical
update runs as torch ops (the reference for tests).
"""
from __future__ import annotations

import math
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from ..ops import weights as W

SSM_LEAVES = {
    "standard": {"B", "Lambda_re", "Lambda_im", "log_step", "norm", "B_bias", "C_bias", "dt_bias", "D"},
    "BandCdecay": {"Lambda_re", "Lambda_im", "log_step", "norm"},
    "BfastandCdecay": {"Lambda_re", "Lambda_im", "log_step", "norm"},
    "noBCdecay": {"B", "C", "C1", "C2", "D", "Lambda_re", "Lambda_im", "log_step", "norm"},
}


def leaf_group(name: str, opt_config: str = "standard", attention_model: bool = False,
               dt_global: bool = False) -> str:
    """``ssm`` (Adam at the ssm lr, no decay) or ``regular`` (AdamW); with ``dt_global`` the
    S5 ``log_step`` moves to the regular group (the reference's ``dt_global`` branch of the
    standard configuration, ``training/train_helpers.py:541-547``)."""
    if attention_model:
        return "regular"
    leaf = name.split(".")[-1]
    if dt_global and leaf == "log_step":
        return "regular"
    return "ssm" if leaf in SSM_LEAVES.get(opt_config, SSM_LEAVES["standard"]) else "regular"


class FlatAdam:
    def __init__(self, model: nn.Module, lr: float, ssm_lr: float, weight_decay: float = 0.05,
                 max_grad_norm: float = 1.0, betas=(0.9, 0.999), eps: float = 1e-8,
                 opt_config: str = "standard", attention_model: bool = False,
                 bf16_shadow: bool = True, pad_multiple: int = 128, alloc=None, last=(), dt_global: bool = False,
                 exclude=()):
        self.model = model
        self.b1, self.b2 = betas
        self.eps = eps
        self.wd = weight_decay
        self.max_grad_norm = max_grad_norm
        self.base_lr = {"ssm": ssm_lr, "regular": lr}
        skip = {id(p) for p in exclude}              # parameters another optimizer owns (FSDP shards)
        named = [(n, p) for n, p in model.named_parameters() if p.requires_grad and id(p) not in skip]
        groups = {"ssm": [], "regular": []}
        for n, p in named:
            groups[leaf_group(n, opt_config, attention_model, dt_global)].append((n, p))
        # parameters in `last` (tensor-parallel slices) go to the end of their group, so each
        # group's slices form one contiguous range [tail_lo[group], group end)
        late = {id(p) for p in last}
        for k in groups:
            groups[k] = [x for x in groups[k] if id(x[1]) not in late] + [x for x in groups[k] if id(x[1]) in late]
        order = groups["ssm"] + groups["regular"]
        dev = order[0][1].device
        # every slice starts on a 128-element boundary so bf16/fp32 views are 256-byte
        # aligned (cuBLAS picks its vectorised kernels only for aligned operands)
        A = 128
        rnd = lambda n: (n + A - 1) // A * A
        total = sum(rnd(p.numel()) for _, p in order)
        total = -(-total // pad_multiple) * pad_multiple   # equal shards when sharded
        self.n_ssm = sum(rnd(p.numel()) for _, p in groups["ssm"])
        self.numel = total
        self.device = dev
        mk = alloc or (lambda n, dt, d: torch.zeros(n, dtype=dt, device=d))
        self.flat = mk(total, torch.float32, dev)
        self.grad = mk(total, torch.float32, dev)
        self.m = torch.zeros(total, dtype=torch.float32, device=dev)
        self.v = torch.zeros(total, dtype=torch.float32, device=dev)
        self.shadow = mk(total, torch.bfloat16, dev) if (bf16_shadow and dev.type == "cuda") else None
        self.names: List[str] = []
        self.slices: Dict[str, Tuple[int, int]] = {}
        self.late_ranges: List[Tuple[int, int]] = []     # [lo, hi) of the `last` parameters per group
        ends = {"ssm": self.n_ssm, "regular": total}
        off = 0
        seen_late = set()
        for n, p in order:
            g = "ssm" if off < self.n_ssm else "regular"
            if id(p) in late and g not in seen_late:
                seen_late.add(g)
                self.late_ranges.append((off, ends[g]))
            k = p.numel()
            self.flat[off:off + k].copy_(p.detach().reshape(-1))
            p.data = self.flat[off:off + k].view_as(p)
            p.grad = self.grad[off:off + k].view_as(p)
            p._s0_flat_grad = True      # fused weight-gradient GEMMs may accumulate into p.grad
            if self.shadow is not None:
                W.register(p, self.shadow[off:off + k].view(p.shape))
            self.names.append(n)
            self.slices[n] = (off, off + k)
            off += rnd(k)
        if self.shadow is not None:
            self.shadow.copy_(self.flat)
        self.step_count = 0
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._lr = torch.zeros(2, dtype=torch.float32, device=dev)
        self.last_grad_norm: Optional[torch.Tensor] = None

    # -- sharding (ZeRO-1/2: each rank owns a contiguous slice of the flat buffer) -------------
    def shard(self, world: int, rank: int) -> None:
        """Keep Adam moments only for this rank's shard ``[lo, hi)`` of the flat buffer
        (``numel / world`` elements; the buffer is padded so the shards are equal)."""
        if self.numel % (128 * world):
            raise ValueError("build FlatAdam with pad_multiple=128*world to shard it")
        per = self.numel // world
        self.world, self.rank = world, rank
        self.shard_per = per
        self.lo, self.hi = min(rank * per, self.numel), min((rank + 1) * per, self.numel)
        n = self.hi - self.lo
        self.m = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.v = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.sharded = True

    def shard_bounds(self):
        if not getattr(self, "sharded", False):
            return None
        return [[min(k * self.shard_per, self.numel), min((k + 1) * self.shard_per, self.numel)]
                for k in range(self.world)]

    def local_moments(self):
        return self.m, self.v

    def load_full_moments(self, m: torch.Tensor, v: torch.Tensor, step: int) -> None:
        """Moments of the whole flat buffer (any sharding at save time) -> this rank's layout."""
        self.step_count = int(step)
        lo, hi = (self.lo, self.hi) if getattr(self, "sharded", False) else (0, self.numel)
        self.m.copy_(m[lo:hi])
        self.v.copy_(v[lo:hi])

    def params_in_order(self):
        named = dict(self.model.named_parameters())
        return [named[n] for n in self.names]

    def refresh_shadow(self):
        if self.shadow is not None:
            self.shadow.copy_(self.flat)

    def zero_grad(self):
        self.grad.zero_()

    def state_dict(self):
        return {"step": self.step_count, "m": self.m, "v": self.v}

    def load_state_dict(self, sd):
        self.step_count = int(sd["step"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])

    def step_shard(self, gshard: torch.Tensor, grad_sumsq: torch.Tensor, lr_scale: float = 1.0) -> None:
        """Adam on this rank's shard only: ``gshard`` is the reduced gradient of ``[lo, hi)``
        and ``grad_sumsq`` the global sum of squares (for clipping)."""
        self.step_count += 1
        t = self.step_count
        bc1, bc2 = 1 - self.b1 ** t, 1 - self.b2 ** t
        lr_s, lr_r = self.base_lr["ssm"] * lr_scale, self.base_lr["regular"] * lr_scale
        self.last_grad_norm = grad_sumsq
        lo, hi, ns = self.lo, self.hi, self.n_ssm
        pieces = []
        if lo < min(hi, ns):
            pieces.append((lo, min(hi, ns), lr_s, 0.0, 0))
        if max(lo, ns) < hi:
            pieces.append((max(lo, ns), hi, lr_r, self.wd, 1))
        if self.device.type == "cuda":
            from ..ops._ext import ext
            C = ext()
            self._lr.copy_(torch.tensor([lr_s, lr_r]), non_blocking=True)
            for a, b, _, wd, gi in pieces:
                sh = self.shadow[a:b] if self.shadow is not None else None
                C.adam(self.flat[a:b], gshard[a - lo:b - lo], self.m[a - lo:b - lo], self.v[a - lo:b - lo], sh,
                       grad_sumsq, self.max_grad_norm, self._lr[gi:gi + 1], self.b1, self.b2, self.eps, wd, bc1, bc2)
            return
        nrm = math.sqrt(float(grad_sumsq))
        scale = 1.0 if (self.max_grad_norm <= 0 or nrm < self.max_grad_norm) else self.max_grad_norm / nrm
        for a, b, lr, wd, _ in pieces:
            g = gshard[a - lo:b - lo] * scale
            m, v, p = self.m[a - lo:b - lo], self.v[a - lo:b - lo], self.flat[a:b]
            m.mul_(self.b1).add_(g, alpha=1 - self.b1)
            v.mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
            p.sub_(lr * ((m / bc1) / ((v / bc2).sqrt() + self.eps) + wd * p))

    def group_grad_norms(self) -> Dict[str, float]:
        """L2 norm of this rank's gradient buffer per optimizer group (ssm / regular), as the
        reference logs grad norms by group (``training/train_helpers.py:290``)."""
        out = {}
        for name, (a, b) in (("ssm", (0, self.n_ssm)), ("regular", (self.n_ssm, self.numel))):
            if b > a:
                out[name] = float(self.grad[a:b].float().norm())
        return out

    def step(self, lr_scale: float = 1.0, grad_sumsq: Optional[torch.Tensor] = None):
        """One update.  ``grad_sumsq`` overrides the local sum of squares (sharded optimizers)."""
        self.step_count += 1
        t = self.step_count
        bc1, bc2 = 1 - self.b1 ** t, 1 - self.b2 ** t
        lr_s, lr_r = self.base_lr["ssm"] * lr_scale, self.base_lr["regular"] * lr_scale
        if self.device.type == "cuda":
            from ..ops._ext import ext
            C = ext()
            if grad_sumsq is None:
                self._sumsq.zero_()
                C.sumsq(self.grad, self._sumsq)
                grad_sumsq = self._sumsq
            self.last_grad_norm = grad_sumsq
            self._lr.copy_(torch.tensor([lr_s, lr_r]), non_blocking=True)
            ns = self.n_ssm
            sh = self.shadow
            if ns:
                C.adam(self.flat[:ns], self.grad[:ns], self.m[:ns], self.v[:ns],
                       sh[:ns] if sh is not None else None, grad_sumsq, self.max_grad_norm,
                       self._lr[0:1], self.b1, self.b2, self.eps, 0.0, bc1, bc2)
            if ns < self.numel:
                C.adam(self.flat[ns:], self.grad[ns:], self.m[ns:], self.v[ns:],
                       sh[ns:] if sh is not None else None, grad_sumsq, self.max_grad_norm,
                       self._lr[1:2], self.b1, self.b2, self.eps, self.wd, bc1, bc2)
            return
        # CPU reference path
        if grad_sumsq is None:
            grad_sumsq = (self.grad * self.grad).sum()
        self.last_grad_norm = grad_sumsq
        nrm = math.sqrt(float(grad_sumsq))
        scale = 1.0 if (self.max_grad_norm <= 0 or nrm < self.max_grad_norm) else self.max_grad_norm / nrm
        for lo, hi, lr, wd in ((0, self.n_ssm, lr_s, 0.0), (self.n_ssm, self.numel, lr_r, self.wd)):
            if lo == hi:
                continue
            g = self.grad[lo:hi] * scale
            m, v, p = self.m[lo:hi], self.v[lo:hi], self.flat[lo:hi]
            m.mul_(self.b1).add_(g, alpha=1 - self.b1)
            v.mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
            upd = (m / bc1) / ((v / bc2).sqrt() + self.eps) + wd * p
            p.sub_(lr * upd)


def cosine_schedule(step: int, warmup_steps: int, total_steps: int, lr_min_frac: float = 0.0) -> float:
    """Linear warmup from 0, then cosine decay to ``lr_min_frac`` (a multiple of the base lr).

    Same shape as the reference's ``create_learning_rate_schedule``
    (``training/train_helpers.py:156-200``), returned as a scale on the base lr.
    """
    if warmup_steps > 0 and step < warmup_steps:
        return step / warmup_steps
    n = max(total_steps - warmup_steps, 1)
    pct = min((step - warmup_steps) / n, 1.0)
    return (1 - lr_min_frac) * 0.5 * (1 + math.cos(math.pi * pct)) + lr_min_frac
