"""Post-training of the state model: five ways to put a preference into the flow.

Same trainer family and call signatures as the reference's
``state/posttraining/{refl,flow_grpo,awm,ram,dmd}.py``; the published methods:

* ``ReFLTrainer`` (reward feedback learning): no-grad Euler prefix from noise down
  to a random late time t in ``t_range``, one graded velocity evaluation, the
  one-jump clean estimate x0_hat = x_t - t v, loss = -reward(x0_hat) (+ an
  optional flow-matching anchor on real data).
* ``FlowGRPOTrainer`` (Flow-GRPO / DanceGRPO): G stochastic (SDE) rollouts of one
  context, group-normalised advantages of a black-box reward, a PPO-clipped
  ratio of per-step Gaussian transition likelihoods on a random subset
  (``timestep_fraction``) of the chain.
* ``AWMTrainer`` (advantage-weighted matching): ODE rollouts, the same group
  advantages (clipped), and the plain flow-matching loss on the rollouts weighted
  by the advantage at ``n_noise_draws`` noise levels (+ optional anchor on real
  windows).
* ``RAMTrainer`` (reward-adjusted matching): the regression target's endpoint
  moves toward the reward-softmax centroid of the group by
  ``beta * (1 - min-max normalised reward)``; the noised input stays the raw rollout.
* ``DMDTrainer`` / ``DMDRTrainer`` (distribution matching distillation): a few-step
  student rollout (Self-Forcing over ``n_blocks`` blocks with ``rebind``), noised to
  a random level; the student's pseudo-loss has gradient (s_fake - s_real) / norm
  with scores of a frozen teacher and an online fake critic (refreshed by flow
  matching on the detached rollouts); DMDR adds a differentiable reward term.

Every trainer returns a dict with the loss tensor(s) to backpropagate and a few
detached diagnostics; optimiser steps stay with the caller.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch

from .flow import (ModelFn, PinFn, RectifiedFlow, fm_loss, interpolate, score_from_v, velocity_target,
                   x0_from_v)

Reward = Callable[[torch.Tensor], torch.Tensor]


def _identity(x):
    return x


def group_advantage(r: torch.Tensor, eps: float = 1e-4, clip: Optional[float] = None) -> torch.Tensor:
    """(r - mean) / (population std + eps), optionally clipped to [-clip, clip]."""
    a = (r - r.mean()) / (r.std(unbiased=False) + eps)
    return a if clip is None else a.clamp(-clip, clip)


def _expand_mask(mask: Optional[torch.Tensor], n: int) -> Optional[torch.Tensor]:
    if mask is None or mask.dim() != 1:
        return mask
    return mask[None].expand(n, -1)


def _anchor_loss(model_fn: ModelFn, data: torch.Tensor, generator=None) -> torch.Tensor:
    """Plain flow-matching loss on real windows (keeps the model on the data manifold)."""
    t = torch.rand(data.shape[0], device=data.device)
    eps = torch.randn(data.shape, device=data.device, generator=generator)
    return fm_loss(model_fn(interpolate(data, eps, t), t), velocity_target(data, eps))


class _GroupTrainer:
    """Shared state of the group methods (one context, G rollouts, one scalar each)."""

    def __init__(self, model_fn: ModelFn, flow: RectifiedFlow, reward: Reward, decode=None,
                 group_size: int = 8):
        if group_size < 2:
            raise ValueError("group_size must be >= 2 to compare rollouts within a group")
        self.model_fn, self.flow, self.reward = model_fn, flow, reward
        self.decode = decode or _identity
        self.group_size = group_size

    def _score(self, x0: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            return self.reward(self.decode(x0))


class ReFLTrainer:
    def __init__(self, model_fn: ModelFn, flow: RectifiedFlow, reward: Reward, decode=None,
                 fm_weight: float = 0.1, t_range=(0.05, 0.4)):
        lo, hi = t_range
        if not 0.0 <= lo < hi <= 1.0:
            raise ValueError(f"t_range must satisfy 0 <= lo < hi <= 1, got {t_range}")
        self.model_fn, self.flow, self.reward = model_fn, flow, reward
        self.decode = decode or _identity
        self.fm_weight, self.t_range = fm_weight, (lo, hi)

    @torch.no_grad()
    def _prefix(self, shape, device, t_stop: float, generator=None) -> torch.Tensor:
        x = torch.randn(shape, device=device, generator=generator)
        for t_val, dt in self.flow._grid():
            if t_val <= t_stop:
                break
            x = x - dt * self.model_fn(x, torch.full((shape[0],), t_val, device=device, dtype=x.dtype))
        return x

    def step(self, shape, device, data_batch: Optional[torch.Tensor] = None, generator=None) -> dict:
        lo, hi = self.t_range
        t_mid = lo + (hi - lo) * float(torch.rand(()))
        x_t = self._prefix(shape, device, t_mid, generator)
        t = torch.full((shape[0],), t_mid, device=device, dtype=x_t.dtype)
        x0_hat = x0_from_v(x_t, self.model_fn(x_t, t), t)
        r = self.reward(self.decode(x0_hat))
        loss = -r.mean()
        anchor = torch.zeros((), device=device)
        if self.fm_weight > 0.0 and data_batch is not None:
            anchor = _anchor_loss(self.model_fn, data_batch)
            loss = loss + self.fm_weight * anchor
        return {"loss": loss, "reward_mean": r.detach().mean(), "fm_anchor": anchor.detach(), "t_mid": t_mid}


class FlowGRPOTrainer(_GroupTrainer):
    def __init__(self, model_fn: ModelFn, flow: RectifiedFlow, reward: Reward, decode=None,
                 group_size: int = 8, clip_range: float = 0.2, timestep_fraction: float = 0.25,
                 adv_eps: float = 1e-4):
        if flow.noise_scale <= 0.0:
            raise ValueError("Flow-GRPO needs a stochastic sampler (RectifiedFlow(noise_scale > 0))")
        if not 0.0 < timestep_fraction <= 1.0:
            raise ValueError("timestep_fraction must be in (0, 1]")
        super().__init__(model_fn, flow, reward, decode, group_size)
        self.clip_range, self.timestep_fraction, self.adv_eps = clip_range, timestep_fraction, adv_eps

    @torch.no_grad()
    def rollout_group(self, frame_shape, device, pin: Optional[PinFn] = None, generator=None):
        return self.flow.sample_sde_trajectory(self.model_fn, (self.group_size, *frame_shape), device,
                                               generator=generator, pin=pin)

    def step(self, frame_shape, device, pin: Optional[PinFn] = None,
             frame_mask: Optional[torch.Tensor] = None, generator=None) -> dict:
        if pin is not None and frame_mask is None:
            raise ValueError("a pinned rollout needs frame_mask (pinned frames are not policy samples)")
        x0, recs = self.rollout_group(frame_shape, device, pin, generator)
        r = self._score(x0)
        adv = group_advantage(r, self.adv_eps)
        n_keep = max(1, round(len(recs) * self.timestep_fraction))
        keep = torch.randperm(len(recs), generator=generator)[:n_keep].tolist()
        mask = _expand_mask(frame_mask, self.group_size)
        terms, ratios = [], []
        for i in keep:
            lp = self.flow.step_log_prob(self.model_fn, recs[i], frame_mask=mask)
            ratio = torch.exp(lp - lp.detach())        # behaviour policy = current policy at rollout time
            lo, hi = 1.0 - self.clip_range, 1.0 + self.clip_range
            terms.append(-torch.minimum(ratio * adv, ratio.clamp(lo, hi) * adv).mean())
            ratios.append(ratio.detach().mean())
        return {"loss": torch.stack(terms).mean(), "reward_mean": r.mean(), "reward_std": r.std(unbiased=False),
                "advantage_abs": adv.abs().mean(), "ratio_mean": torch.stack(ratios).mean(),
                "kept_transitions": n_keep}


class AWMTrainer(_GroupTrainer):
    def __init__(self, model_fn: ModelFn, flow: RectifiedFlow, reward: Reward, decode=None,
                 group_size: int = 8, n_noise_draws: int = 4, adv_clip: float = 3.0, adv_eps: float = 1e-4,
                 fm_anchor_weight: float = 0.0):
        if n_noise_draws < 1:
            raise ValueError("n_noise_draws must be >= 1")
        super().__init__(model_fn, flow, reward, decode, group_size)
        self.n_noise_draws, self.adv_clip, self.adv_eps = n_noise_draws, adv_clip, adv_eps
        self.fm_anchor_weight = fm_anchor_weight

    def step(self, frame_shape, device, pin: Optional[PinFn] = None,
             frame_mask: Optional[torch.Tensor] = None, data_batch: Optional[torch.Tensor] = None,
             generator=None) -> dict:
        G = self.group_size
        x0 = self.flow.sample_ode(self.model_fn, (G, *frame_shape), device, generator=generator, pin=pin)
        r = self._score(x0)
        adv = group_advantage(r, self.adv_eps, self.adv_clip)
        mask = _expand_mask(frame_mask, G)
        draws = []
        for _ in range(self.n_noise_draws):
            t = torch.rand(G, device=device)
            eps = torch.randn(x0.shape, device=device, generator=generator)
            draws.append(fm_loss(self.model_fn(interpolate(x0, eps, t), t), velocity_target(x0, eps),
                                 weight=adv, frame_mask=mask))
        loss = torch.stack(draws).mean()
        anchor = torch.zeros((), device=device)
        if self.fm_anchor_weight > 0.0 and data_batch is not None:
            anchor = _anchor_loss(self.model_fn, data_batch, generator)
            loss = loss + self.fm_anchor_weight * anchor
        return {"loss": loss, "reward_mean": r.mean(), "reward_std": r.std(unbiased=False),
                "advantage_abs": adv.abs().mean(), "fm_anchor": anchor.detach()}


class RAMTrainer(_GroupTrainer):
    def __init__(self, model_fn: ModelFn, flow: RectifiedFlow, reward: Reward, decode=None,
                 group_size: int = 8, n_noise_draws: int = 4, beta: float = 1.0, temperature: float = 0.5):
        if not 0.0 <= beta <= 1.0:
            raise ValueError("beta must be in [0, 1]")
        super().__init__(model_fn, flow, reward, decode, group_size)
        self.n_noise_draws, self.beta, self.temperature = n_noise_draws, beta, temperature

    @torch.no_grad()
    def adjusted_endpoints(self, x0: torch.Tensor, r: torch.Tensor):
        """(x0_adj, r_tilde): endpoints pulled toward the reward-softmax centroid."""
        r_tilde = (r - r.min()) / (r.max() - r.min()).clamp_min(1e-8)
        shape = (-1,) + (1,) * (x0.dim() - 1)
        centroid = (torch.softmax(r / self.temperature, 0).view(shape) * x0).sum(0, keepdim=True)
        w = (self.beta * (1.0 - r_tilde)).view(shape)
        return x0 + w * (centroid - x0), r_tilde

    def step(self, frame_shape, device, pin: Optional[PinFn] = None,
             frame_mask: Optional[torch.Tensor] = None, generator=None) -> dict:
        G = self.group_size
        x0 = self.flow.sample_ode(self.model_fn, (G, *frame_shape), device, generator=generator, pin=pin)
        r = self._score(x0)
        x0_adj, r_tilde = self.adjusted_endpoints(x0, r)
        mask = _expand_mask(frame_mask, G)
        draws = []
        for _ in range(self.n_noise_draws):
            t = torch.rand(G, device=device)
            eps = torch.randn(x0.shape, device=device, generator=generator)
            draws.append(fm_loss(self.model_fn(interpolate(x0, eps, t), t), velocity_target(x0_adj, eps),
                                 frame_mask=mask))
        return {"loss": torch.stack(draws).mean(), "reward_mean": r.mean(),
                "endpoint_shift": (x0_adj - x0).abs().mean(), "r_tilde_mean": r_tilde.mean()}


class DMDTrainer:
    def __init__(self, student_fn: ModelFn, teacher_fn: ModelFn, fake_fn: ModelFn, flow: RectifiedFlow,
                 student_steps: int = 4, n_blocks: int = 1, t_range=(0.02, 0.98),
                 rebind: Optional[Callable[[torch.Tensor], ModelFn]] = None):
        if n_blocks > 1 and rebind is None:
            raise ValueError("multi-block Self-Forcing needs rebind(previous_block) -> ModelFn")
        self.student_fn, self.teacher_fn, self.fake_fn, self.flow = student_fn, teacher_fn, fake_fn, flow
        self.student_steps, self.n_blocks, self.t_range, self.rebind = student_steps, n_blocks, t_range, rebind

    def _few_step(self, fn: ModelFn, shape, device, generator=None) -> torch.Tensor:
        """Few-step Euler with gradients (the student is what trains)."""
        x = torch.randn(shape, device=device, generator=generator)
        n = self.student_steps
        for i in range(n):
            x = x - (1.0 / n) * fn(x, torch.full((shape[0],), 1.0 - i / n, device=device, dtype=x.dtype))
        return x

    def rollout(self, shape, device, generator=None) -> torch.Tensor:
        blocks: List[torch.Tensor] = []
        fn = self.student_fn
        for _ in range(self.n_blocks):
            blk = self._few_step(fn, shape, device, generator)
            blocks.append(blk)
            if self.rebind is not None:
                fn = self.rebind(blk.detach())        # condition the next block on generated history
        return blocks[0] if len(blocks) == 1 else torch.cat(blocks, 1)

    def step(self, frame_shape, device, batch_size: int = 8, generator=None) -> dict:
        x_gen = self.rollout((batch_size, *frame_shape), device, generator)
        lo, hi = self.t_range
        t = lo + (hi - lo) * torch.rand(batch_size, device=device)
        x_t = interpolate(x_gen, torch.randn(x_gen.shape, device=device, generator=generator), t)
        with torch.no_grad():
            v_real = self.teacher_fn(x_t, t)
            gap = score_from_v(x_t, self.fake_fn(x_t, t), t) - score_from_v(x_t, v_real, t)
            norm = (x_gen - x0_from_v(x_t, v_real, t)).abs().flatten(1).mean(1).clamp_min(1e-4)
            norm = norm.view(-1, *([1] * (x_gen.dim() - 1)))
        loss_student = (x_gen * (gap / norm)).mean()          # d/dx_gen = gap / norm (per element / numel)
        xd = x_gen.detach()
        t_c = torch.rand(batch_size, device=device)
        eps_c = torch.randn(xd.shape, device=device, generator=generator)
        loss_fake = fm_loss(self.fake_fn(interpolate(xd, eps_c, t_c), t_c), velocity_target(xd, eps_c))
        return {"loss_student": loss_student, "loss_fake": loss_fake, "score_gap": gap.abs().mean(),
                "x_gen": x_gen}


class DMDRTrainer(DMDTrainer):
    """DMD plus a differentiable reward on the same student rollout."""

    def __init__(self, *args, reward: Reward, decode=None, reward_weight: float = 1.0, **kwargs):
        super().__init__(*args, **kwargs)
        self.reward, self.decode, self.reward_weight = reward, decode or _identity, reward_weight

    def step(self, frame_shape, device, batch_size: int = 8, generator=None) -> dict:
        out = super().step(frame_shape, device, batch_size, generator)
        r = self.reward(self.decode(out["x_gen"]))
        out["loss_student"] = out["loss_student"] - self.reward_weight * r.mean()
        out["reward_mean"] = r.detach().mean()
        return out
