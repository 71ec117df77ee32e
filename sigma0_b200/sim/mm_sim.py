"""Closed-loop market-making simulator: a quoting policy against a frozen episode.

Two worlds answer "what happens to our quotes" (the reference's heuristic-learning
simulator, ``post_training/heuristic_learning/mm_sim.py:151``,
``episode_builder.py:219``, ``fidelity.py:261,324``, ``autopsy.py:131``):

* ``replay``: the episode's real continuation is replayed through the book with our
  orders inserted -- our orders fill against real flow, but the flow does not react;
* ``generator``: the world model, conditioned on the episode's context, generates
  the continuation message by message with our orders resting in the same book,
  so the generated flow sees them through the book state (interventional
  ``p(market | do(our quotes))``); our fills are settled by the engine, never by the
  model.

``autopsy`` splits an episode's PnL into spread capture (fill price vs the mid at
the fill) and inventory revaluation, plus fill counts and the final inventory.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

from ..envs.lob_env import AGENT_OID_BASE, BaseLOBEnv, EnvWindow, MarketMakingEnv


@dataclass
class Episode:
    context_tokens: torch.Tensor   # (L,) START-shifted context tokens
    context_books: torch.Tensor    # (n_ctx, d_book)
    last_token: int
    l2_start: np.ndarray           # book before the context
    context_msgs: np.ndarray       # (n_ctx, 8) engine rows of the context
    future_msgs: np.ndarray        # (n_future, 8) real continuation
    t_start: tuple


def build_episodes(days, tokenizer, n_ctx: int, n_future: int) -> List[Episode]:
    from ..data.book_transform import transform_books_numpy
    from ..encoding import START_TOK
    out = []
    for d in days:
        for s in range(0, d.msgs.shape[0] - n_ctx - n_future + 1, n_ctx + n_future):
            t = tokenizer.encode_msgs(d.msgs[s:s + n_ctx]).reshape(-1)
            out.append(Episode(torch.from_numpy(np.concatenate([[START_TOK], t[:-1]])),
                               torch.from_numpy(transform_books_numpy(d.books[s:s + n_ctx]).astype(np.float32)),
                               int(t[-1]), np.asarray(d.books[s, 3:], np.int64), d.engine_msgs[s:s + n_ctx],
                               d.engine_msgs[s + n_ctx:s + n_ctx + n_future], (int(d.books[s, 1]), 0)))
    return out


@dataclass
class EpisodeResult:
    pnl_ticks: np.ndarray
    inventory: np.ndarray
    spread_capture_ticks: np.ndarray
    n_fills: np.ndarray
    steps: int
    log: List[Dict] = field(default_factory=list)


def _fill_stats(trades: torch.Tensor, tid: int, mid: torch.Tensor):
    q, cash = BaseLOBEnv.fills(trades, tid)
    price = trades[..., 0].double()
    valid = trades[..., 0] >= 0
    mine = valid & ((trades[..., 6] == tid) | (trades[..., 7] == tid))
    signed = torch.where(trades[..., 7] == tid, -trades[..., 1], trades[..., 1]).double()
    capture = ((mid.double()[:, None] - price) * signed * mine).sum(-1)   # bought below / sold above the mid
    return q, cash, capture, mine.sum(-1)


def run_episodes(policy: Callable, episodes: List[Episode], world: str = "replay", model=None,
                 token_mode: str = "22tok", steps: int = 10, msgs_per_step: int = 2, quote_size: int = 100,
                 device="cpu", seed: int = 0) -> EpisodeResult:
    """Run ``policy(obs, env) -> (n, 1, 2) offset indices`` on every episode in parallel."""
    n = len(episodes)
    helper = MarketMakingEnv([EnvWindow(e.future_msgs, e.l2_start, e.t_start) for e in episodes], n_envs=n,
                             msgs_per_step=msgs_per_step, quote_size=quote_size, device=device, seed=seed)
    tid = helper.tids[0]
    inv = torch.zeros(n, dtype=torch.long)
    cash = torch.zeros(n, dtype=torch.float64)
    capture = torch.zeros(n, dtype=torch.float64)
    fills = torch.zeros(n, dtype=torch.long)
    log = []
    if world == "replay":
        # book = context replayed, then the real continuation with our orders in it
        helper.reset(list(range(n)))
        ctx = torch.from_numpy(np.stack([e.context_msgs for e in episodes]).astype(np.int32))
        helper.engine.process(ctx if not helper.engine.on_gpu else ctx.to(helper.engine.device))
        helper.max_steps = min(steps, helper.max_steps)
        obs = helper._obs(helper.observe())
        for t in range(helper.max_steps):
            act = policy(obs, helper)
            trades, _ = helper.step_messages(helper.action_messages(act, obs["mid"]))
            q, c, cap, nf = _fill_stats(trades, tid, obs["mid"])
            inv += q; cash += c.double(); capture += cap; fills += nf
            helper.inv[:, 0] = inv
            obs = helper._obs(helper.observe())
            log.append({"step": t, "mean_inventory": float(inv.double().mean())})
        mid = obs["mid"].double()
    elif world == "generator":
        from ..infer import Generator
        gen = Generator(model, token_mode, top_n=-1, seed=seed, use_graphs=False)
        gen.condition(torch.stack([e.context_tokens for e in episodes]), torch.stack([e.context_books for e in episodes]),
                      torch.tensor([e.last_token for e in episodes]), np.stack([e.l2_start for e in episodes]),
                      np.stack([e.context_msgs for e in episodes]), start_time=episodes[0].t_start)
        helper.reset(list(range(n)))
        helper.max_steps = steps

        def observe():
            asks, bids = gen.sides()
            a = asks[:, :, 0].clone()
            a[a < 0] = 2**31 - 1
            ba = a.min(1).values
            bb = bids[:, :, 0].max(1).values
            ok = (ba < 2**31 - 1) & (bb > 0)
            mid = torch.where(ok, (ba + bb) // 2 // helper.tick * helper.tick, gen.p_mid.cpu().long())
            return {"mid": mid, "inventory": inv[:, None].clone(), "time_left": torch.full((n,), 1.0),
                    "spread": torch.where(ok, (ba - bb) // helper.tick, torch.zeros_like(ba)),
                    "imbalance": torch.zeros(n), "l2": torch.zeros(n, 40, dtype=torch.long)}

        # our quote bookkeeping lives in the helper; the book is the generator's
        helper.engine.sides = lambda: tuple(x.numpy() for x in gen.sides())
        obs = observe()
        for t in range(steps):
            obs["time_left"] = torch.full((n,), float(steps - t) / steps)
            act = policy(obs, helper)
            msgs = helper.action_messages(act, obs["mid"])
            ts = gen.time.cpu()
            msgs[:, :, 6], msgs[:, :, 7] = ts[:, None, 0], ts[:, None, 1]
            gen.apply_engine_messages(msgs)
            gen.generate(msgs_per_step)
            trades = gen.trade_rows()
            q, c, cap, nf = _fill_stats(trades, tid, obs["mid"])
            inv += q; cash += c.double(); capture += cap; fills += nf
            obs = observe()
            log.append({"step": t, "mean_inventory": float(inv.double().mean())})
        mid = obs["mid"].double()
    else:
        raise ValueError(f"world must be 'replay' or 'generator', not {world!r}")
    pnl = (cash + inv.double() * mid) / helper.tick
    return EpisodeResult(pnl.numpy(), inv.numpy(), (capture / helper.tick).numpy(), fills.numpy(),
                         len(log), log)


def autopsy(res: EpisodeResult) -> Dict[str, float]:
    """Episode PnL split: spread capture + inventory revaluation (= the rest)."""
    return {"pnl_ticks_mean": float(res.pnl_ticks.mean()),
            "spread_capture_ticks_mean": float(res.spread_capture_ticks.mean()),
            "inventory_pnl_ticks_mean": float((res.pnl_ticks - res.spread_capture_ticks).mean()),
            "fills_mean": float(res.n_fills.mean()), "abs_final_inventory_mean": float(np.abs(res.inventory).mean())}
