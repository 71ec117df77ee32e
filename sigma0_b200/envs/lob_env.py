"""Batched limit-order-book environments on the matching engine.

The reference builds gymnax environments on its JAX engine: a base environment
that replays LOBSTER windows (``environment/jaxen/base_env.py:84-230``), a
market-making agent (``mm_env.py:151``), an optimal-execution agent
(``exec_env.py:143``) and a multi-agent environment sharing one book
(``marl_env.py:45``).  Here every environment of a batch is one book of the
batched engine (``engine/batched.py``: one warp per book on the GPU, the numpy
oracle on the CPU), so thousands of environments step in one kernel launch.

Per step each environment:
1. applies the agents' messages (cancels and new orders, each tagged with the
   agent's trader id),
2. replays the next ``msgs_per_step`` messages of its data window,
3. reads the trades of the step and attributes fills to agents by trader id
   (as aggressor: ``-qty`` column sign; as resting order: ``+qty``),
4. returns the L2 state.

``MarketMakingEnv`` quotes one bid and one ask per step at ``mid -/+ offset``
ticks (discrete offsets), replacing the previous quotes; reward = change of
mark-to-market PnL minus an inventory penalty.  ``ExecutionEnv`` must buy (or
sell) a target quantity within the episode; actions choose a child-order size,
sent as a marketable order; reward = negative implementation shortfall against
the arrival mid.  ``MultiAgentEnv`` runs several market makers and an executor
on the same books.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from ..engine.batched import BatchedEngine
from ..engine.book import EngineConfig, init_msgs_from_l2

AGENT_OID_BASE = 100_000_000


@dataclass
class EnvWindow:
    engine_msgs: np.ndarray    # (n, 8) data messages
    l2_start: np.ndarray       # (4L,) book before the first message
    t0: tuple                  # (sec, ns) of the first message


def windows_from_days(days, length: int, stride: Optional[int] = None) -> List[EnvWindow]:
    out = []
    for d in days:
        n = d.engine_msgs.shape[0]
        for s in range(0, n - length + 1, stride or length):
            out.append(EnvWindow(d.engine_msgs[s:s + length], np.asarray(d.books[s, 3:], np.int64),
                                 (int(d.books[s, 1]), int(d.books[s, 2]))))
    return out


class BaseLOBEnv:
    """Replays data windows through batched books; agents add their own messages."""

    def __init__(self, windows: Sequence[EnvWindow], n_envs: int, msgs_per_step: int = 5, n_agents: int = 0,
                 cfg: EngineConfig = EngineConfig(n_trades=128, n_orders=128), device="cpu", tick: int = 100,
                 seed: int = 0):
        self.windows, self.n, self.k = list(windows), n_envs, msgs_per_step
        self.n_agents, self.cfg, self.tick = n_agents, cfg, tick
        self.dev = torch.device(device)
        self.rng = np.random.default_rng(seed)
        self.engine = BatchedEngine(n_envs, cfg, device=device)
        L = min(w.engine_msgs.shape[0] for w in self.windows)
        self.max_steps = L // msgs_per_step

    # -- episode control ------------------------------------------------------------------
    def reset(self, idx: Optional[Sequence[int]] = None):
        if idx is None:
            idx = self.rng.integers(len(self.windows), size=self.n)
        self.idx = np.asarray(idx)
        ws = [self.windows[i] for i in self.idx]
        self.engine.reset()
        init = np.stack([init_msgs_from_l2(w.l2_start, self.cfg, w.t0) for w in ws])
        self.engine.process(init)
        T = self.max_steps * self.k
        self.data = torch.from_numpy(np.stack([w.engine_msgs[:T] for w in ws]).astype(np.int32))
        self.t = 0
        self.clock = torch.from_numpy(np.array([w.t0 for w in ws], dtype=np.int64))
        self._clear_trades()
        return self.observe()

    def _clear_trades(self):
        if self.engine.on_gpu:
            self.engine.trades.fill_(-1)
        else:
            for ob in self.engine.books:
                ob.trades[:] = -1

    # -- stepping ----------------------------------------------------------------------------
    def step_messages(self, agent_msgs: Optional[torch.Tensor]):
        """agent_msgs (n, m, 8) or None; returns (trades (n, n_trades, 8) int64, data msgs of the step)."""
        self._clear_trades()
        data = self.data[:, self.t * self.k:(self.t + 1) * self.k]
        # agent messages take the timestamp of the step's first data message
        if agent_msgs is not None and agent_msgs.shape[1]:
            am = agent_msgs.clone().to(torch.int32).cpu()
            am[:, :, 6] = data[:, :1, 6]
            am[:, :, 7] = data[:, :1, 7]
            msgs = torch.cat([am, data], 1)
        else:
            msgs = data
        self.engine.process(msgs.to(self.engine.device) if self.engine.on_gpu else msgs)
        self.t += 1
        self.clock = data[:, -1, 6:8].long()
        return torch.from_numpy(self.engine.trade_rows()), data

    def observe(self) -> Dict[str, torch.Tensor]:
        l2 = self.engine.l2(10).long().cpu()
        ap, av, bp, bv = l2[:, 0], l2[:, 1], l2[:, 2], l2[:, 3]
        ok = (ap < 2**31 - 1) & (bp > -(2**31 - 1))
        mid = torch.where(ok, (ap + bp) // 2 // self.tick * self.tick, torch.zeros_like(ap))   # tick-floored
        spread = torch.where(ok, (ap - bp) // self.tick, torch.zeros_like(ap))
        imb = (bv - av).float() / (bv + av).clamp(min=1).float()
        return {"l2": l2, "mid": mid, "spread": spread, "imbalance": imb,
                "time_left": torch.full((self.n,), float(self.max_steps - self.t) / self.max_steps)}

    @property
    def done(self) -> bool:
        return self.t >= self.max_steps

    @staticmethod
    def fills(trades: torch.Tensor, tid: int):
        """Signed filled quantity (+ bought) and cash flow of trader ``tid`` per env."""
        price, q = trades[..., 0], trades[..., 1]
        valid = trades[..., 0] >= 0
        aggr = valid & (trades[..., 7] == tid)
        pas = valid & (trades[..., 6] == tid)
        signed = torch.where(aggr, -q, torch.zeros_like(q)) + torch.where(pas, q, torch.zeros_like(q))
        return signed.sum(-1), -(signed * price).sum(-1)


class MarketMakingEnv(BaseLOBEnv):
    """One (or several) market makers quoting around the mid each step."""

    OFFSETS = (1, 2, 3, 5, 8)

    def __init__(self, *a, quote_size: int = 100, inventory_penalty: float = 0.01, n_mm: int = 1, **kw):
        super().__init__(*a, n_agents=n_mm, **kw)
        self.size, self.pen, self.n_mm = quote_size, inventory_penalty, n_mm
        self.tids = [1000 + i for i in range(n_mm)]

    def reset(self, idx=None):
        obs = super().reset(idx)
        z = lambda: torch.zeros(self.n, self.n_mm, dtype=torch.long)
        self.inv, self.cash = z(), z().double()
        self.live = torch.zeros(self.n, self.n_mm, 2, 2, dtype=torch.long)   # [side][oid, price]
        self.seq = 0
        self.pnl_prev = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        return self._obs(obs)

    def _obs(self, o):
        o = dict(o)
        o["inventory"] = self.inv.clone()
        return o

    def action_messages(self, actions: torch.Tensor, mid: torch.Tensor) -> torch.Tensor:
        """actions (n, n_mm, 2) offset indices (bid, ask) -> (n, 4*n_mm, 8) messages."""
        msgs = []
        off = torch.tensor(self.OFFSETS)
        asks, bids = self.engine.sides()
        resting = {0: torch.from_numpy(bids[:, :, 2]), 1: torch.from_numpy(asks[:, :, 2])}
        for a in range(self.n_mm):
            tid = self.tids[a]
            for side in (0, 1):        # 0 bid, 1 ask
                oid, price = self.live[:, a, side, 0], self.live[:, a, side, 1]
                # cancel only quotes still resting: a failed lookup would hit the engine's
                # last-row fallback and disturb someone else's order
                alive = (resting[side] == oid[:, None]).any(1) & (oid != 0)
                oid = torch.where(alive, oid, torch.zeros_like(oid))
                cancel = torch.stack([torch.full_like(oid, 3), torch.full_like(oid, 1 if side == 0 else -1),
                                      torch.full_like(oid, 10**9), price, oid, torch.full_like(oid, tid),
                                      torch.zeros_like(oid), torch.zeros_like(oid)], -1)
                cancel[oid == 0] = 0                                  # nothing live yet: no-op row
                msgs.append(cancel)
            self.seq += 1
            for side in (0, 1):
                d = off[actions[:, a, side]] * self.tick
                price = mid - d if side == 0 else mid + d
                oid = torch.full_like(mid, AGENT_OID_BASE + (a * 2 + side) * 10**6 + self.seq)
                new = torch.stack([torch.ones_like(mid), torch.full_like(mid, 1 if side == 0 else -1),
                                   torch.full_like(mid, self.size), price, oid, torch.full_like(mid, tid),
                                   torch.zeros_like(mid), torch.zeros_like(mid)], -1)
                new[mid <= 0] = 0
                msgs.append(new)
                self.live[:, a, side, 0] = torch.where(mid > 0, oid, torch.zeros_like(oid))
                self.live[:, a, side, 1] = price
        return torch.stack(msgs, 1)

    def step(self, actions: torch.Tensor):
        obs0 = self.observe()
        trades, _ = self.step_messages(self.action_messages(actions, obs0["mid"]))
        obs = self.observe()
        rew = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        for a, tid in enumerate(self.tids):
            q, c = self.fills(trades, tid)
            self.inv[:, a] += q
            self.cash[:, a] += c.double()
            pnl = self.cash[:, a] + self.inv[:, a].double() * obs["mid"].double()
            rew[:, a] = (pnl - self.pnl_prev[:, a]) / self.tick - self.pen * self.inv[:, a].double().abs()
            self.pnl_prev[:, a] = pnl
        return self._obs(obs), rew, self.done


class ExecutionEnv(BaseLOBEnv):
    """Buy (side=1) or sell (side=0) ``target`` shares before the episode ends."""

    SIZES = (0, 50, 100, 200, 400)

    def __init__(self, *a, target: int = 1000, side: int = 1, **kw):
        super().__init__(*a, n_agents=1, **kw)
        self.target, self.side, self.tid = target, side, 2000

    def reset(self, idx=None):
        o = super().reset(idx)
        self.done_qty = torch.zeros(self.n, dtype=torch.long)
        self.cash = torch.zeros(self.n, dtype=torch.float64)
        self.arrival = o["mid"].clone()
        self.seq = 0
        o["remaining"] = torch.full((self.n,), self.target)
        return o

    def step(self, actions: torch.Tensor):
        """actions (n,) size indices; the last step sweeps what is left."""
        rem = self.target - self.done_qty
        q = torch.tensor(self.SIZES)[actions].clamp(max=rem)
        if self.t == self.max_steps - 1:
            q = rem
        self.seq += 1
        sgn = 1 if self.side == 1 else -1
        far = torch.full_like(q, 10**9 if self.side == 1 else 1)
        oid = torch.full_like(q, AGENT_OID_BASE + 50 * 10**6 + self.seq)
        m = torch.stack([torch.full_like(q, 4), torch.full_like(q, -sgn), q, far, oid, torch.full_like(q, self.tid),
                         torch.zeros_like(q), torch.zeros_like(q)], -1)[:, None]
        # type 4 is the execution of a resting order on the *opposite* side: side flag is the
        # resting side, so a buy execution hits the ask side (-1)
        m[q <= 0] = 0
        trades, _ = self.step_messages(m)
        filled, cash = self.fills(trades, self.tid)
        filled = filled * sgn
        self.done_qty += filled
        self.cash += cash.double()
        o = self.observe()
        # shortfall vs arrival mid, in ticks per share
        avg_px = (-self.cash * sgn) / self.done_qty.clamp(min=1).double()
        short = (avg_px - self.arrival.double()) * sgn / self.tick
        rew = torch.where(filled > 0, -short * filled.double() / self.target, torch.zeros_like(short))
        o["remaining"] = self.target - self.done_qty
        return o, rew, self.done


class MultiAgentEnv(MarketMakingEnv):
    """Several market makers (and optionally an executor) trading on the same books."""

    def __init__(self, *a, n_mm: int = 2, exec_target: int = 0, **kw):
        super().__init__(*a, n_mm=n_mm, **kw)
        self.exec_target = exec_target
        self.exec_tid = 2000

    def step(self, actions: torch.Tensor, exec_qty: Optional[torch.Tensor] = None):
        obs0 = self.observe()
        msgs = self.action_messages(actions, obs0["mid"])
        if exec_qty is not None:
            q = exec_qty.long()
            m = torch.stack([torch.full_like(q, 4), torch.full_like(q, -1), q, torch.full_like(q, 10**9),
                             torch.full_like(q, AGENT_OID_BASE + 60 * 10**6 + self.t), torch.full_like(q, self.exec_tid),
                             torch.zeros_like(q), torch.zeros_like(q)], -1)[:, None]
            m[q <= 0] = 0
            msgs = torch.cat([msgs, m], 1)
        trades, _ = self.step_messages(msgs)
        obs = self.observe()
        rew = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        for a, tid in enumerate(self.tids):
            q, c = self.fills(trades, tid)
            self.inv[:, a] += q
            self.cash[:, a] += c.double()
            pnl = self.cash[:, a] + self.inv[:, a].double() * obs["mid"].double()
            rew[:, a] = (pnl - self.pnl_prev[:, a]) / self.tick - self.pen * self.inv[:, a].double().abs()
            self.pnl_prev[:, a] = pnl
        return self._obs(obs), rew, self.done


def features(obs: Dict[str, torch.Tensor], n_agents: int = 1) -> torch.Tensor:
    """Per-agent observation vector: spread, imbalance, time left, inventory, top-5 level volumes."""
    l2 = obs["l2"].double()
    vols = torch.stack([l2[:, 4 * i + 1] for i in range(5)] + [l2[:, 4 * i + 3] for i in range(5)], -1) / 1000.0
    base = torch.cat([obs["spread"].double()[:, None], obs["imbalance"].double()[:, None],
                      obs["time_left"].double()[:, None], vols], -1)
    inv = obs.get("inventory")
    inv = inv.double() / 1000.0 if inv is not None else torch.zeros(l2.shape[0], n_agents, dtype=torch.float64)
    return torch.cat([base[:, None].expand(-1, inv.shape[1], -1), inv[..., None]], -1).float()
