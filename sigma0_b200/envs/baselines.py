"""Market-making baselines and a policy evaluator.

* ``avellaneda_stoikov``: reservation price ``r = s - q * gamma * sigma^2 * tau`` and
  total spread ``gamma * sigma^2 * tau + (2 / gamma) * ln(1 + gamma / kappa)``
  (Avellaneda & Stoikov, "High-frequency trading in a limit order book", 2008),
  mapped onto the environment's discrete quote offsets;
* ``fixed_offset``: constant quote offsets;
* ``MultiplicativeWeights``: the one-armed-bandit market maker of the reference
  (``environment/jaxrl/market_making_baselines/MMMW_baseline.py``): weights over a
  discrete action set, an action drawn in proportion to them, and after each step the
  drawn action's weight multiplied by ``exp(eta * reward)`` and the weights renormalised
  (here per environment and agent, all environments of a batch at once);
* ``evaluate``: mean episode PnL, inventory and fill statistics of a policy
  (the reference's ``jaxrl/MARL/baseline_eval`` and ``market_making_baselines``).
"""
from __future__ import annotations

import math
from typing import Callable, Dict

import numpy as np
import torch


def _nearest_offset_index(ticks: torch.Tensor, offsets) -> torch.Tensor:
    o = torch.tensor(offsets, dtype=torch.float64)
    return (ticks.double()[..., None] - o).abs().argmin(-1)


def avellaneda_stoikov(gamma: float = 0.1, sigma_ticks: float = 2.0, kappa: float = 1.5, inv_scale: float = 100.0):
    def policy(obs, env) -> torch.Tensor:
        tau = obs["time_left"].double()[:, None]
        q = obs["inventory"].double() / inv_scale
        skew = q * gamma * sigma_ticks ** 2 * tau                       # reservation shift, ticks
        half = 0.5 * (gamma * sigma_ticks ** 2 * tau + (2.0 / gamma) * math.log(1 + gamma / kappa))
        bid = (half + skew).clamp(min=1.0)
        ask = (half - skew).clamp(min=1.0)
        return torch.stack([_nearest_offset_index(bid, env.OFFSETS), _nearest_offset_index(ask, env.OFFSETS)], -1)
    return policy


def fixed_offset(bid_idx: int = 1, ask_idx: int = 1):
    def policy(obs, env) -> torch.Tensor:
        n, a = obs["inventory"].shape
        return torch.tensor([bid_idx, ask_idx]).expand(n, a, 2).clone()
    return policy


def evaluate(env, policy: Callable, episodes: int = 1) -> Dict[str, float]:
    pnl, inv, rews = [], [], []
    for _ in range(episodes):
        obs = env.reset()
        total = torch.zeros(env.n, env.n_mm, dtype=torch.float64)
        while not env.done:
            obs, r, _ = env.step(policy(obs, env))
            total += r
        pnl.append((env.pnl_prev / env.tick).numpy())
        inv.append(env.inv.numpy())
        rews.append(total.numpy())
    pnl, inv, rews = np.concatenate(pnl), np.concatenate(inv), np.concatenate(rews)
    return {"pnl_ticks_mean": float(pnl.mean()), "pnl_ticks_std": float(pnl.std()),
            "abs_inventory_mean": float(np.abs(inv).mean()), "reward_mean": float(rews.mean())}


class MultiplicativeWeights:
    """Multiplicative-weights action selection over ``n_actions`` discrete actions, one
    weight vector per (environment, agent)."""

    def __init__(self, n_actions: int, eta: float = 0.1, n_envs: int = 1, n_agents: int = 1, seed: int = 0):
        self.eta = eta
        self.w = torch.full((n_envs, n_agents, n_actions), 1.0 / n_actions, dtype=torch.float64)
        self.gen = torch.Generator().manual_seed(seed)
        self.last: torch.Tensor = torch.zeros(n_envs, n_agents, dtype=torch.long)

    def policy(self, obs=None, env=None) -> torch.Tensor:
        n, a, k = self.w.shape
        self.last = torch.multinomial(self.w.reshape(n * a, k), 1, generator=self.gen).reshape(n, a)
        return self.last.clone()

    def update(self, reward: torch.Tensor) -> None:
        """Scale the weight of the action drawn last by exp(eta * reward) and renormalise; the
        exponent is clipped so one huge reward cannot underflow every other weight."""
        r = reward.double().reshape(self.last.shape)
        f = torch.exp((self.eta * r).clamp(-50.0, 50.0))
        self.w.scatter_(-1, self.last[..., None], self.w.gather(-1, self.last[..., None]) * f[..., None])
        self.w /= self.w.sum(-1, keepdim=True)


def run_bandit(env, bandit: MultiplicativeWeights, episodes: int = 1) -> Dict[str, float]:
    """Episodes of ``env`` with actions from ``bandit``, updated after every step."""
    rews = []
    for _ in range(episodes):
        env.reset()
        total = torch.zeros(env.n, env.n_mm, dtype=torch.float64)
        while not env.done:
            _, r, _ = env.step(bandit.policy())
            bandit.update(r)
            total += r
        rews.append(total.numpy())
    rews = np.concatenate(rews)
    return {"reward_mean": float(rews.mean()), "weights_max_mean": float(bandit.w.max(-1).values.mean())}
