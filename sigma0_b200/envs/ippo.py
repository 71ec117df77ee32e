"""Independent PPO with recurrent (GRU) actor-critics for the LOB agents.

The reference trains IPPO over its JAX multi-agent environment
(``environment/jaxrl/MARL/ippo_rnn_JAXMARL.py``; data-parallel with ``pmean`` in
``..._pmap.py:567-568,789``): one GRU actor-critic per agent TYPE (market makers and
executors each keep their own network, optimizer, learning rate, gradient clip and learning-
rate annealing, ``:383-425,525-545``), shared by every agent of that type; multi-discrete
actions through independent categorical heads or autoregressive ones where head k also sees
the actions already drawn (``MultiActionOutputIndependant`` / ``...Autoregressive``,
``:81-200``); GAE(lambda), the clipped objective over minibatches and epochs.

Here the same structure runs on the batched-engine environments: ``MarketMakingEnv`` (one
market-maker type), ``ExecutionEnv`` (one executor) and ``MultiAgentEnv`` (market makers and
executors on the same books).  The action dimensions come from the environment's configured
action spaces (``action_dims``); observations are the book features of ``lob_env.features``
plus, for executors, the share of the task left and its side.  When a process group is
initialised each rank runs its own environments and the gradients are averaged across ranks
after every backward.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from .lob_env import ExecutionEnv, MultiAgentEnv, features

# multi-discrete action dimensions of every configured action space
MM_DIMS = {"offsets": (5, 5), "bobRL": (5, 3), "spread_skew": (5, 5), "fixed_quants": (8,), "AvSt": (8,),
           "bobStrategy": (5,), "directional_trading": (5,), "simple": (4,)}
EXEC_DIMS = {"sizes": (5,), "fixed_quants": (6,), "fixed_quants_1msg": (5,), "fixed_quants_complex": (13,),
             "simplest_case": (2,), "twap": (1,), "fixed_prices": (3, 3, 3, 3)}


def action_dims(kind: str, space: str, n_levels: int = 3) -> Tuple[int, ...]:
    if kind == "mm":
        return (3,) * (2 * n_levels) if space == "fixed_prices" else MM_DIMS[space]
    return EXEC_DIMS[space]


class GRUActorCritic(nn.Module):
    """GRU trunk, one categorical head per action dimension (autoregressive heads also
    take the one-hot of the dimensions drawn before them), and a value head."""

    def __init__(self, obs_dim: int, dims: Sequence[int], hidden: int = 64, autoregressive: bool = False):
        super().__init__()
        self.dims, self.hidden, self.ar = tuple(dims), hidden, autoregressive
        self.inp = nn.Sequential(nn.Linear(obs_dim, hidden), nn.Tanh())
        self.gru = nn.GRUCell(hidden, hidden)
        extra = [sum(self.dims[:k]) if autoregressive else 0 for k in range(len(self.dims))]
        self.heads = nn.ModuleList([nn.Linear(hidden + e, d) for d, e in zip(self.dims, extra)])
        self.v = nn.Linear(hidden, 1)

    def _dist(self, h, k, prev: List[torch.Tensor]):
        x = h
        if self.ar and k:
            x = torch.cat([h] + [nn.functional.one_hot(a, d).float() for a, d in zip(prev, self.dims)], -1)
        return torch.distributions.Categorical(logits=self.heads[k](x))

    def forward(self, x, h, actions: Optional[torch.Tensor] = None):
        """(actions (B, K), log-prob (B,), entropy (B,), value (B,), new hidden); with
        ``actions`` given their log-probability under the current policy."""
        h = self.gru(self.inp(x), h)
        acts, lp, ent = [], 0.0, 0.0
        for k in range(len(self.dims)):
            d = self._dist(h, k, acts)
            a = d.sample() if actions is None else actions[:, k]
            acts.append(a)
            lp = lp + d.log_prob(a)
            ent = ent + d.entropy()
        return torch.stack(acts, -1), lp, ent, self.v(h)[..., 0], h


# kept for callers of the earlier two-head policy
GRUPolicy = GRUActorCritic


@dataclass
class PPOConfig:
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    lr: float = 3e-4
    epochs: int = 4
    minibatches: int = 1
    ent_coef: float = 0.01
    vf_coef: float = 0.5
    max_grad_norm: float = 0.5
    anneal_lr: bool = False
    hidden: int = 64
    autoregressive: bool = False
    # per agent type overrides of lr / max_grad_norm / anneal_lr, e.g. {"exe": {"lr": 1e-4}}
    per_type: Dict[str, Dict] = field(default_factory=dict)


@dataclass
class _Group:
    name: str
    n_agents: int
    dims: Tuple[int, ...]
    cols: slice                    # its columns of the reward matrix


def _groups(env) -> List[_Group]:
    if isinstance(env, ExecutionEnv):
        return [_Group("exe", 1, action_dims("exe", env.space), slice(0, 1))]
    gs = [_Group("mm", env.n_mm, action_dims("mm", env.space, env.n_levels), slice(0, env.n_mm))]
    if isinstance(env, MultiAgentEnv) and env.n_exec:
        gs.append(_Group("exe", env.n_exec, action_dims("exe", env.exec_space),
                         slice(env.n_mm, env.n_mm + env.n_exec)))
    return gs


def _obs(env, obs, g: _Group) -> torch.Tensor:
    """(n, A, d) observations of group g."""
    if g.name == "mm":
        return features(obs, g.n_agents)
    base = features({k: v for k, v in obs.items() if k != "inventory"}, 1)[:, 0]        # (n, d)
    if isinstance(env, ExecutionEnv):
        left = (obs["remaining"].double() / env.target).float()[:, None]
        side = obs.get("is_sell", torch.zeros(env.n, dtype=torch.bool)).float()[:, None]
    else:
        left = (obs["exec_remaining"].double() / env.exec_target).float()
        side = env.exec_sell.float()
    n, A = base.shape[0], g.n_agents
    return torch.cat([base[:, None].expand(n, A, -1), left.reshape(n, A, 1), side.reshape(n, A, 1)], -1)


def _to_env(a: torch.Tensor, g: _Group, n: int, single: bool) -> torch.Tensor:
    """(n * A, K) sampled actions -> the environment's layout."""
    a = a.reshape(n, g.n_agents, len(g.dims))
    if len(g.dims) == 1:
        a = a[..., 0]
    return a[:, 0] if single else a


def _step(env, acts: Dict[str, torch.Tensor]):
    if isinstance(env, ExecutionEnv):
        obs, r, done = env.step(acts["exe"])
        return obs, r.reshape(env.n, 1), done
    if isinstance(env, MultiAgentEnv) and env.n_exec:
        return env.step(acts["mm"], exec_actions=acts["exe"])
    return env.step(acts["mm"])


def train_ippo(env, iterations: int = 10, cfg: PPOConfig = PPOConfig(), seed: int = 0, log=None):
    """Train one actor-critic per agent type for ``iterations`` episodes of ``env``; returns
    (history, policy) -- the policy of the only type, or a {type: policy} dict."""
    torch.manual_seed(seed)
    groups = _groups(env)
    obs = env.reset()
    world = dist.get_world_size() if dist.is_initialized() else 1
    single = isinstance(env, ExecutionEnv)
    pols, opts, scheds = {}, {}, {}
    for g in groups:
        o = {**{"lr": cfg.lr, "max_grad_norm": cfg.max_grad_norm, "anneal_lr": cfg.anneal_lr},
             **cfg.per_type.get(g.name, {})}
        pols[g.name] = GRUActorCritic(_obs(env, obs, g).shape[-1], g.dims, cfg.hidden, cfg.autoregressive)
        opts[g.name] = torch.optim.Adam(pols[g.name].parameters(), lr=o["lr"], eps=1e-5)
        scheds[g.name] = o
    hist = []
    for it in range(iterations):
        for g in groups:                                   # linear annealing over the iterations
            if scheds[g.name]["anneal_lr"]:
                for pg in opts[g.name].param_groups:
                    pg["lr"] = scheds[g.name]["lr"] * (1.0 - it / max(iterations, 1))
        obs = env.reset()
        n = env.n
        hs = {g.name: torch.zeros(n * g.n_agents, cfg.hidden) for g in groups}
        buf = {g.name: {"x": [], "h": [], "a": [], "lp": [], "v": [], "r": [], "live": [], "end": []}
               for g in groups}
        with torch.no_grad():
            while not env.done:
                # environments of different episode lengths (fixed-time episodes): a finished
                # one is frozen; its samples are left out and its value is not bootstrapped
                alive = ~env.ended if hasattr(env, "ended") else torch.ones(n, dtype=torch.bool)
                acts = {}
                for g in groups:
                    x = _obs(env, obs, g).reshape(n * g.n_agents, -1)
                    a, lp, _, v, h2 = pols[g.name](x, hs[g.name])
                    b = buf[g.name]
                    b["x"].append(x); b["h"].append(hs[g.name]); b["a"].append(a); b["lp"].append(lp)
                    b["v"].append(v)
                    hs[g.name] = h2
                    acts[g.name] = _to_env(a, g, n, single)
                obs, r, _ = _step(env, acts)
                end = env.ended if hasattr(env, "ended") else torch.zeros(n, dtype=torch.bool)
                for g in groups:
                    buf[g.name]["r"].append(r[:, g.cols].reshape(-1).float())
                    buf[g.name]["live"].append(alive[:, None].expand(n, g.n_agents).reshape(-1))
                    buf[g.name]["end"].append(end[:, None].expand(n, g.n_agents).reshape(-1).float())
        rec = {"iteration": it}
        for g in groups:
            b, pol, opt = buf[g.name], pols[g.name], opts[g.name]
            T = len(b["r"])
            vals, rews = torch.stack(b["v"]), torch.stack(b["r"])
            adv = torch.zeros_like(rews)
            last = torch.zeros_like(rews[0])
            ends = torch.stack(b["end"])
            for t in reversed(range(T)):
                cont = 1.0 - ends[t]                       # no bootstrap past an episode's end
                nv = vals[t + 1] * cont if t + 1 < T else torch.zeros_like(vals[t])
                last = rews[t] + cfg.gamma * nv - vals[t] + cfg.gamma * cfg.lam * cont * last
                adv[t] = last
            keep = torch.stack(b["live"]).reshape(-1)
            ret = (adv + vals).reshape(-1)[keep]
            a_k = adv.reshape(-1)[keep]
            advn = (a_k - a_k.mean()) / (a_k.std() + 1e-8)
            X, H = torch.stack(b["x"]).reshape(T * n * g.n_agents, -1)[keep], \
                torch.stack(b["h"]).reshape(-1, cfg.hidden)[keep]
            ACT, LP = torch.stack(b["a"]).reshape(-1, len(g.dims))[keep], torch.stack(b["lp"]).reshape(-1)[keep]
            N = X.shape[0]
            for _ in range(cfg.epochs):
                perm = torch.randperm(N)
                # exactly NUM_MINIBATCHES updates per epoch on every rank (their sample counts
                # differ with fixed-time episodes; the gradient all-reduce needs equal counts)
                for i in torch.tensor_split(perm, max(1, cfg.minibatches)):
                    if i.numel() == 0:
                        loss = sum(p.sum() * 0.0 for p in pol.parameters())
                    else:
                        _, lp, ent, v, _ = pol(X[i], H[i], ACT[i])
                        ratio = torch.exp(lp - LP[i])
                        a = advn[i]
                        pg = -torch.min(ratio * a, ratio.clamp(1 - cfg.clip, 1 + cfg.clip) * a).mean()
                        loss = pg + cfg.vf_coef * ((v - ret[i]) ** 2).mean() - cfg.ent_coef * ent.mean()
                    opt.zero_grad()
                    loss.backward()
                    if world > 1:
                        for p in pol.parameters():
                            if p.grad is not None:
                                dist.all_reduce(p.grad)
                                p.grad.div_(world)
                    nn.utils.clip_grad_norm_(pol.parameters(), scheds[g.name]["max_grad_norm"])
                    opt.step()
            rec[f"{g.name}_mean_return"] = float(rews.sum(0).mean())
            rec[f"{g.name}_loss"] = float(loss.detach())
        # the first type's numbers under the plain keys
        rec["mean_return"], rec["loss"] = rec[f"{groups[0].name}_mean_return"], rec[f"{groups[0].name}_loss"]
        hist.append(rec)
        if log:
            log(rec)
    return hist, (pols[groups[0].name] if len(groups) == 1 else pols)
