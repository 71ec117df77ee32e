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
from typing import Callable, Dict, List, Sequence

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


def fixed_action_sweep(env, fixed_actions: Dict[str, Sequence], episodes: int = 1) -> List[Dict]:
    """Every combination of fixed actions across the agent types: the reference's
    baseline-only evaluation (``environment/jaxrl/MARL/baseline_eval/baseline_only_JAXMARL.py:140-520``,
    a fixed-action network per type; ``plotting_combinations.py`` tabulates the
    combinations).  ``fixed_actions`` maps a type (``mm``, ``exe``) to the actions to try,
    each an int or one int per action dimension; every agent of the type plays it at every
    step.  One row per combination: the actions and, per type, the mean episode return over
    agents, environments and episodes (plus the market makers' mean absolute inventory and
    the executors' mean executed quantity)."""
    import itertools

    from .ippo import _groups, _step
    groups = _groups(env)
    names = [g.name for g in groups]
    missing = [n for n in names if n not in fixed_actions]
    if missing:
        raise ValueError(f"fixed actions needed for the agent types {missing}")
    choices = [[tuple(np.atleast_1d(a).astype(int).tolist()) for a in fixed_actions[n]] for n in names]
    for g, cs in zip(groups, choices):
        for c in cs:
            if len(c) != len(g.dims) or any(not 0 <= x < d for x, d in zip(c, g.dims)):
                raise ValueError(f"action {c} does not fit the {g.name} action dimensions {g.dims}")
    rows = []
    for combo in itertools.product(*choices):
        rets = {n: [] for n in names}
        extra = {"mm_abs_inventory": [], "exe_executed": []}
        for _ in range(episodes):
            env.reset()
            total = None
            while not env.done:
                acts = {}
                for g, c in zip(groups, combo):
                    a = torch.tensor(c, dtype=torch.long).expand(env.n, g.n_agents, len(c))
                    a = a[..., 0] if len(c) == 1 else a
                    acts[g.name] = a[:, 0] if names == ["exe"] else a
                _, r, _ = _step(env, acts)
                total = r.double() if total is None else total + r.double()
            for g in groups:
                rets[g.name].append(total[:, g.cols].mean().item())
            if hasattr(env, "inv"):
                extra["mm_abs_inventory"].append(env.inv.abs().double().mean().item())
            done = getattr(env, "exec_done", getattr(env, "done_qty", None))
            if done is not None and "exe" in names:
                extra["exe_executed"].append(done.double().mean().item())
        row = {f"{n}_action": list(c) for n, c in zip(names, combo)}
        row.update({f"{n}_return": float(np.mean(v)) for n, v in rets.items()})
        row.update({k: float(np.mean(v)) for k, v in extra.items() if v})
        rows.append(row)
    return rows
