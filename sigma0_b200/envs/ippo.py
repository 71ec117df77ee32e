"""Independent PPO with a shared recurrent (GRU) policy for the market-making agents.

The reference trains IPPO with a GRU actor-critic over its JAX multi-agent
environment, data-parallel with ``pmean`` over devices
(``environment/jaxrl/MARL/ippo_rnn_JAXMARL.py``, ``..._pmap.py:567-568,789``).
Here: one policy shared by all agents (agent index is not an input, as in
IPPO with parameter sharing), factorised categorical heads for the bid and ask
offsets, GAE(lambda) advantages, the clipped PPO objective, and -- when a
process group is initialised -- gradient averaging across ranks after every
backward (each rank runs its own batch of environments).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import torch
import torch.distributed as dist
import torch.nn as nn

from .lob_env import features


class GRUPolicy(nn.Module):
    def __init__(self, obs_dim: int, n_actions: int, hidden: int = 64):
        super().__init__()
        self.inp = nn.Sequential(nn.Linear(obs_dim, hidden), nn.Tanh())
        self.gru = nn.GRUCell(hidden, hidden)
        self.bid = nn.Linear(hidden, n_actions)
        self.ask = nn.Linear(hidden, n_actions)
        self.v = nn.Linear(hidden, 1)
        self.hidden = hidden

    def forward(self, x, h):
        h = self.gru(self.inp(x), h)
        return torch.distributions.Categorical(logits=self.bid(h)), torch.distributions.Categorical(
            logits=self.ask(h)), self.v(h)[..., 0], h


@dataclass
class PPOConfig:
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    lr: float = 3e-4
    epochs: int = 4
    ent_coef: float = 0.01
    vf_coef: float = 0.5
    max_grad_norm: float = 0.5


def train_ippo(env, iterations: int = 10, cfg: PPOConfig = PPOConfig(), seed: int = 0, log=None) -> List[Dict]:
    torch.manual_seed(seed)
    obs = env.reset()
    A = env.n_mm
    x0 = features(obs, A)
    pol = GRUPolicy(x0.shape[-1], len(env.OFFSETS))
    opt = torch.optim.Adam(pol.parameters(), lr=cfg.lr)
    world = dist.get_world_size() if dist.is_initialized() else 1
    hist = []
    for it in range(iterations):
        obs = env.reset()
        h = torch.zeros(env.n * A, pol.hidden)
        xs, hs, acts, logps, vals, rews = [], [], [], [], [], []
        with torch.no_grad():
            while not env.done:
                x = features(obs, A).reshape(env.n * A, -1)
                db, da, v, h2 = pol(x, h)
                ab, aa = db.sample(), da.sample()
                xs.append(x); hs.append(h); acts.append(torch.stack([ab, aa], -1))
                logps.append(db.log_prob(ab) + da.log_prob(aa)); vals.append(v)
                obs, r, _ = env.step(torch.stack([ab, aa], -1).reshape(env.n, A, 2))
                rews.append(r.reshape(-1).float())
                h = h2
        T = len(rews)
        adv = torch.zeros(T, env.n * A)
        last = torch.zeros(env.n * A)
        for t in reversed(range(T)):
            nv = vals[t + 1] if t + 1 < T else torch.zeros_like(vals[t])
            delta = rews[t] + cfg.gamma * nv - vals[t]
            last = delta + cfg.gamma * cfg.lam * last
            adv[t] = last
        ret = adv + torch.stack(vals)
        advn = (adv - adv.mean()) / (adv.std() + 1e-8)
        X, H, ACT, LP = torch.stack(xs), torch.stack(hs), torch.stack(acts), torch.stack(logps)
        for _ in range(cfg.epochs):
            db, da, v, _ = pol(X.reshape(T * env.n * A, -1), H.reshape(T * env.n * A, -1))
            lp = db.log_prob(ACT[..., 0].reshape(-1)) + da.log_prob(ACT[..., 1].reshape(-1))
            ratio = torch.exp(lp - LP.reshape(-1))
            a = advn.reshape(-1)
            pg = -torch.min(ratio * a, ratio.clamp(1 - cfg.clip, 1 + cfg.clip) * a).mean()
            vl = ((v - ret.reshape(-1)) ** 2).mean()
            ent = (db.entropy() + da.entropy()).mean()
            loss = pg + cfg.vf_coef * vl - cfg.ent_coef * ent
            opt.zero_grad()
            loss.backward()
            if world > 1:
                for p in pol.parameters():
                    if p.grad is not None:
                        dist.all_reduce(p.grad)
                        p.grad.div_(world)
            nn.utils.clip_grad_norm_(pol.parameters(), cfg.max_grad_norm)
            opt.step()
        rec = {"iteration": it, "mean_return": float(torch.stack(rews).sum(0).mean()), "loss": float(loss)}
        hist.append(rec)
        if log:
            log(rec)
    return hist, pol
