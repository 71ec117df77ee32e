"""Rectified flow for the state model: interpolation, losses, ODE/SDE samplers.

Convention (the reference's ``state/flow.py``, kept so numbers and checkpoints
carry over): t = 0 is data, t = 1 is noise,

    x_t = (1 - t) x0 + t eps,      target velocity v* = eps - x0,

and sampling integrates from t = 1 to t = 0 with ``x <- x - dt v``.  Given a
predicted velocity v at (x_t, t):

    x0_hat  = x_t - t v            (clean estimate)
    eps_hat = x_t + (1 - t) v      (noise estimate)
    score   = -eps_hat / t         (Tweedie for the Gaussian path with sigma_t = t)

The exploration sampler is the marginal-preserving reverse SDE
``dx = [v - sigma_t^2/2 * score] dt + sigma_t dW`` (Euler-Maruyama), with
``sigma_t = a sqrt(t / (1 - t))``; its Gaussian transitions give the per-step
log-likelihoods that Flow-GRPO ratios need.  With ``a = 0`` every step is the
Euler ODE step.

A ``ModelFn`` is ``fn(x_t (B, L, C), t (B,)) -> v``; conditioning is bound inside
it (``dit.bind_condition``).  A ``PinFn`` ``pin(x, t_next)`` re-imposes known
frames after each sampler step (RePaint-style inpainting).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch

ModelFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]
PinFn = Callable[[torch.Tensor, float], torch.Tensor]
T_FLOOR = 1e-4      # below this t the 1/t of the score is not used (deterministic step)


def _bt(t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """(B,) -> broadcastable against ``like`` (B, ...)."""
    return t.reshape(-1, *([1] * (like.dim() - 1))).to(like.dtype)


def interpolate(x0, eps, t):
    tb = _bt(t, x0)
    return x0 + tb * (eps - x0)


def velocity_target(x0, eps):
    return eps - x0


def x0_from_v(x_t, v, t):
    return x_t - _bt(t, x_t) * v


def eps_from_v(x_t, v, t):
    return x_t + (1.0 - _bt(t, x_t)) * v


def score_from_v(x_t, v, t):
    tb = _bt(t, x_t).clamp_min(T_FLOOR)
    return -(x_t + (1.0 - tb) * v) / tb


def fm_loss(v_pred, v_target, *, weight: Optional[torch.Tensor] = None,
            frame_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mean over samples of the per-sample MSE; ``frame_mask`` (B, L) restricts each
    sample's mean to its generated frames, ``weight`` (B,) scales each sample (may be
    negative: advantage weighting)."""
    sq = (v_pred - v_target).square()
    if frame_mask is None:
        per = sq.flatten(1).mean(1)
    else:
        m = frame_mask.to(sq.dtype)[..., None].expand_as(sq)
        per = (sq * m).flatten(1).sum(1) / m.flatten(1).sum(1).clamp_min(1.0)
    if weight is not None:
        per = per * weight.to(per.dtype)
    return per.mean()


@dataclass
class SdeStepRecord:
    """One sampler transition x_t -> x_s (s = t - dt), enough to recompute its log-prob."""
    x_t: torch.Tensor
    x_s: torch.Tensor
    t: torch.Tensor          # (B,)
    dt: float
    noise_std: float         # sigma_t sqrt(dt); 0 for a deterministic step


class RectifiedFlow:
    def __init__(self, num_steps: int = 50, noise_scale: float = 0.0):
        if num_steps < 1:
            raise ValueError("num_steps must be >= 1")
        self.num_steps, self.noise_scale = num_steps, noise_scale

    def timesteps(self, device=None) -> torch.Tensor:
        return torch.linspace(1.0, 0.0, self.num_steps + 1, device=device)

    def _grid(self) -> List[Tuple[float, float]]:
        """(t, dt) of every step, as Python floats (no device syncs)."""
        n = self.num_steps
        return [(1.0 - i / n, 1.0 / n) for i in range(n)]

    def sigma(self, t: float) -> float:
        if self.noise_scale == 0.0:
            return 0.0
        tc = min(max(t, 0.0), 1.0 - 1e-3)
        return self.noise_scale * math.sqrt(tc / (1.0 - tc))

    def drift(self, model_fn: ModelFn, x_t, t, sigma_t: float):
        v = model_fn(x_t, t)
        if sigma_t == 0.0:
            return v
        return v - (0.5 * sigma_t * sigma_t) * score_from_v(x_t, v, t)

    def sde_step(self, model_fn: ModelFn, x_t, t_val: float, dt: float, generator=None) -> SdeStepRecord:
        t = torch.full((x_t.shape[0],), t_val, device=x_t.device, dtype=x_t.dtype)
        sig = self.sigma(t_val) if t_val > T_FLOOR else 0.0
        with torch.no_grad():
            mean = x_t - dt * self.drift(model_fn, x_t, t, sig)
        std = sig * math.sqrt(dt)
        if std > 0.0:
            x_s = mean + std * torch.randn(x_t.shape, device=x_t.device, dtype=x_t.dtype, generator=generator)
        else:
            x_s = mean
        return SdeStepRecord(x_t, x_s, t, dt, std)

    def step_log_prob(self, model_fn: ModelFn, rec: SdeStepRecord,
                      frame_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Differentiable log N(x_s; mean_theta(x_t), noise_std^2) summed per sample."""
        if rec.noise_std <= 0.0:
            raise ValueError("the transition is deterministic; sample with noise_scale > 0")
        sig = self.sigma(float(rec.t[0]))
        mean = rec.x_t - rec.dt * self.drift(model_fn, rec.x_t, rec.t, sig)
        var = rec.noise_std ** 2
        lp = -0.5 * (rec.x_s - mean).square() / var - 0.5 * math.log(2.0 * math.pi * var)
        if frame_mask is not None:
            lp = lp * frame_mask.to(lp.dtype)[..., None]
        return lp.flatten(1).sum(1)

    @torch.no_grad()
    def sample_ode(self, model_fn: ModelFn, shape, device, generator=None, pin: Optional[PinFn] = None):
        x = torch.randn(shape, device=device, generator=generator)
        for t_val, dt in self._grid():
            t = torch.full((shape[0],), t_val, device=device, dtype=x.dtype)
            x = x - dt * model_fn(x, t)
            if pin is not None:
                x = pin(x, t_val - dt)
        return x

    def sample_sde_trajectory(self, model_fn: ModelFn, shape, device, generator=None,
                              pin: Optional[PinFn] = None):
        """(x0, records): a stochastic rollout keeping every transition.  With a pin
        the pinned frames are not Gaussian draws: mask them out of ``step_log_prob``."""
        x = torch.randn(shape, device=device, generator=generator)
        recs: List[SdeStepRecord] = []
        for t_val, dt in self._grid():
            r = self.sde_step(model_fn, x, t_val, dt, generator)
            if pin is not None:
                r = SdeStepRecord(r.x_t, pin(r.x_s, t_val - dt), r.t, r.dt, r.noise_std)
            recs.append(r)
            x = r.x_s
        return x, recs


def make_repaint_pin(x_obs: torch.Tensor, obs_mask: torch.Tensor, generator=None) -> PinFn:
    """Replace observed frames (obs_mask (B, L) == 1) by their forward-noised true
    values at the next sampler time; generated frames pass through."""
    m = obs_mask.to(x_obs.dtype)
    if m.dim() == 2:
        m = m[..., None]

    def pin(x: torch.Tensor, t_next: float) -> torch.Tensor:
        noise = torch.randn(x_obs.shape, device=x_obs.device, dtype=x_obs.dtype, generator=generator)
        return x + m * ((1.0 - t_next) * x_obs + t_next * noise - x)

    return pin
