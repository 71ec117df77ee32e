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
mark-to-market PnL minus an inventory penalty.  The reference's other options are
keywords (or its config field names through ``from_reference_config``): the action
spaces and rewards of ``envs/agents.py``, the end-of-episode unwind of the remaining
inventory at the mid / average mid / far touch with a penalty in ticks, auto-liquidation
above an inventory threshold, reward clipping, the market-share volume bonus, zero
reward while the spread is extreme, and the ``basic`` / ``engineered`` observation
vectors (``agent_observation``).  ``ExecutionEnv`` must buy (or
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


def windows_from_days(days, length: int, stride: Optional[int] = None, ep_type: str = "fixed_steps",
                      msgs_per_step: int = 1) -> List[EnvWindow]:
    """Episode windows of the days' message streams, each with the book before its first
    message.  ``fixed_steps``: ``length`` messages every ``stride`` (default ``length``).
    ``fixed_time``: the messages of consecutive ``length``-second intervals from the day's
    first second, each cut to a whole number of ``msgs_per_step`` steps (intervals with less
    than one step are left out), so windows differ in length (the reference's
    ``matching_engine/jaxlobster/lobster_loader.py:415-490``)."""
    if ep_type not in ("fixed_steps", "fixed_time"):
        raise ValueError("ep_type is fixed_steps or fixed_time")
    out = []
    for d in days:
        msgs = d.engine_msgs
        n = msgs.shape[0]
        if ep_type == "fixed_steps":
            starts = [(s, s + length) for s in range(0, n - length + 1, stride or length)]
        else:
            sec = msgs[:, 6].astype(np.int64)
            edges = np.arange(int(sec[0]), int(sec[-1]) + 1 + length, length)
            cut = np.searchsorted(sec, edges, side="left")
            starts = []
            for lo, hi in zip(cut[:-1], cut[1:]):
                hi = lo + (hi - lo) // msgs_per_step * msgs_per_step
                if hi > lo:
                    starts.append((int(lo), int(hi)))
        for s, e in starts:
            out.append(EnvWindow(msgs[s:e], np.asarray(d.books[s, 3:], np.int64),
                                 (int(d.books[s, 1]), int(d.books[s, 2]))))
    return out


class BaseLOBEnv:
    """Replays data windows through batched books; agents add their own messages.

    ``ep_type="fixed_steps"`` (default): every episode runs the same number of steps, the
    shortest window's.  ``ep_type="fixed_time"``: the windows are ``episode_time``-second
    intervals of different lengths (``windows_from_days(..., ep_type="fixed_time")``); each
    environment runs its own window's steps, ``time_left`` is the fraction of
    ``episode_time`` left on the data clock, an environment whose window has run out is
    frozen (no data, its agents' messages dropped, zero reward) until all have ended, and its
    last step comes at the end of its window or once at most ``last_step_seconds`` are left
    (the reference's ``exec_env.py:1350-1356``)."""

    def __init__(self, windows: Sequence[EnvWindow], n_envs: int, msgs_per_step: int = 5, n_agents: int = 0,
                 cfg: EngineConfig = EngineConfig(n_trades=128, n_orders=128), device="cpu", tick: int = 100,
                 seed: int = 0, ep_type: str = "fixed_steps", episode_time: Optional[float] = None,
                 last_step_seconds: float = 5.0):
        if ep_type not in ("fixed_steps", "fixed_time"):
            raise ValueError("ep_type is fixed_steps or fixed_time")
        if ep_type == "fixed_time" and not episode_time:
            raise ValueError("fixed_time episodes need episode_time (seconds)")
        self.windows, self.n, self.k = list(windows), n_envs, msgs_per_step
        self.n_agents, self.cfg, self.tick = n_agents, cfg, tick
        self.ep_type, self.episode_time, self.last_step_seconds = ep_type, episode_time, last_step_seconds
        self.dev = torch.device(device)
        self.rng = np.random.default_rng(seed)
        self.engine = BatchedEngine(n_envs, cfg, device=device)
        lens = [w.engine_msgs.shape[0] for w in self.windows]
        self.max_steps = (max(lens) if ep_type == "fixed_time" else min(lens)) // msgs_per_step
        self.steps_env = torch.full((n_envs,), self.max_steps, dtype=torch.long)

    # -- episode control ------------------------------------------------------------------
    def reset(self, idx: Optional[Sequence[int]] = None):
        if idx is None:
            idx = self.rng.integers(len(self.windows), size=self.n)
        self.idx = np.asarray(idx)
        ws = [self.windows[i] for i in self.idx]
        self.engine.reset()
        init = np.stack([init_msgs_from_l2(w.l2_start, self.cfg, w.t0) for w in ws])
        self.engine.process(init)
        if self.ep_type == "fixed_time":
            self.steps_env = torch.tensor([w.engine_msgs.shape[0] // self.k for w in ws], dtype=torch.long)
            T = int(self.steps_env.max()) * self.k
            data = np.zeros((self.n, T, 8), np.int32)          # zero rows are no-ops
            for i, w in enumerate(ws):
                m = int(self.steps_env[i]) * self.k
                data[i, :m] = w.engine_msgs[:m]
            self.data = torch.from_numpy(data)
        else:
            T = self.max_steps * self.k
            self.data = torch.from_numpy(np.stack([w.engine_msgs[:T] for w in ws]).astype(np.int32))
        self.t = 0
        self.last_data = torch.zeros(self.n, self.k, 8, dtype=torch.int32)
        self.clock = torch.from_numpy(np.array([w.t0 for w in ws], dtype=np.int64))
        self.t_start = self.clock.clone()
        self.prev_ended = torch.zeros(self.n, dtype=torch.bool)
        self._clear_trades()
        return self.observe()

    def elapsed_seconds(self) -> torch.Tensor:
        """(n,) data-clock seconds since each episode's first message."""
        d = self.clock - self.t_start
        return d[:, 0].double() + d[:, 1].double() * 1e-9

    def time_left(self) -> torch.Tensor:
        """(n,) fraction of the episode left: steps for ``fixed_steps``, the data clock
        against ``episode_time`` for ``fixed_time``."""
        if self.ep_type == "fixed_time":
            return ((self.episode_time - self.elapsed_seconds()) / self.episode_time).clamp(0.0, 1.0).float()
        return torch.full((self.n,), float(self.max_steps - self.t) / self.max_steps)

    def steps_left(self) -> torch.Tensor:
        """(n,) steps left in each environment's episode, this one included."""
        return (self.steps_env - self.t).clamp(min=0)

    def last_step(self) -> torch.Tensor:
        """(n,) True where the coming step is the episode's last."""
        last = self.steps_env - self.t == 1
        if self.ep_type == "fixed_time":
            live = self.t < self.steps_env
            last |= live & (self.episode_time - self.elapsed_seconds() <= self.last_step_seconds)
        return last

    @property
    def ended(self) -> torch.Tensor:
        """(n,) True for environments whose episode is over."""
        return self.t >= self.steps_env

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
        over = self.ended
        self.prev_ended = over
        # agent messages take the timestamp of the step's first data message
        if agent_msgs is not None and agent_msgs.shape[1]:
            am = agent_msgs.clone().to(torch.int32).cpu()
            am[:, :, 6] = data[:, :1, 6]
            am[:, :, 7] = data[:, :1, 7]
            am[over] = 0                                    # a finished episode stays frozen
            msgs = torch.cat([am, data], 1)
        else:
            msgs = data
        self.engine.process(msgs.to(self.engine.device) if self.engine.on_gpu else msgs)
        self.last_data = data
        self.t += 1
        self.clock = torch.where(over[:, None], self.clock, data[:, -1, 6:8].long())
        return torch.from_numpy(self.engine.trade_rows()), data

    def observe(self) -> Dict[str, torch.Tensor]:
        l2 = self.engine.l2(10).long().cpu()
        ap, av, bp, bv = l2[:, 0], l2[:, 1], l2[:, 2], l2[:, 3]
        ok = (ap < 2**31 - 1) & (bp > -(2**31 - 1))
        mid = torch.where(ok, (ap + bp) // 2 // self.tick * self.tick, torch.zeros_like(ap))   # tick-floored
        spread = torch.where(ok, (ap - bp) // self.tick, torch.zeros_like(ap))
        imb = (bv - av).float() / (bv + av).clamp(min=1).float()
        # an empty side of the book makes the step's prices meaningless: the reference reports
        # it as abort_episode (marl_env.py:360) and so does every observation here
        return {"l2": l2, "mid": mid, "spread": spread, "imbalance": imb, "abort_episode": ~ok,
                "time_left": self.time_left()}

    @property
    def done(self) -> bool:
        return bool(self.ended.all())

    @staticmethod
    def fills(trades: torch.Tensor, tid: int):
        """Signed filled quantity (+ bought) and cash flow of trader ``tid`` per env."""
        price, q = trades[..., 0], trades[..., 1]
        valid = trades[..., 0] >= 0
        aggr = valid & (trades[..., 7] == tid)
        pas = valid & (trades[..., 6] == tid)
        signed = torch.where(aggr, -q, torch.zeros_like(q)) + torch.where(pas, q, torch.zeros_like(q))
        return signed.sum(-1), -(signed * price).sum(-1)


class _Quoting:
    """Order management shared by the agents: each agent keeps up to K resting orders; a
    step cancels those still resting and submits the new set (``envs/agents.py``)."""

    def _init_live(self, n_agents: int, K: int):
        self.live = torch.zeros(self.n, n_agents, K, 3, dtype=torch.long)   # (oid, side, price)
        self.seq = 0

    def _order_messages(self, a: int, tid: int, orders: torch.Tensor, market: Optional[torch.Tensor] = None,
                        oid_block: int = 0) -> List[torch.Tensor]:
        """Rows (n, 8) cancelling agent a's resting orders and placing ``orders`` (n, K, 3)
        and the marketable ``market`` (n, 2) = (side, qty)."""
        asks, bids = self.engine.sides()
        in_b, in_a = torch.from_numpy(bids[:, :, 2]), torch.from_numpy(asks[:, :, 2])
        rows = []
        K = self.live.shape[2]
        for k in range(K):
            oid, side, price = self.live[:, a, k, 0], self.live[:, a, k, 1], self.live[:, a, k, 2]
            resting = torch.where(side > 0, (in_b == oid[:, None]).any(1), (in_a == oid[:, None]).any(1))
            # cancel only orders still resting: a failed lookup would fall back to another order
            ok = resting & (oid != 0)
            c = torch.stack([torch.full_like(oid, 3), torch.where(side > 0, 1, -1), torch.full_like(oid, 10**9),
                             price, oid, torch.full_like(oid, tid), torch.zeros_like(oid), torch.zeros_like(oid)], -1)
            c[~ok] = 0
            rows.append(c)
        self.seq += 1
        self.live[:, a] = 0
        for k in range(orders.shape[1]):
            side, price, qty = orders[:, k, 0], orders[:, k, 1], orders[:, k, 2]
            oid = torch.full_like(qty, AGENT_OID_BASE + (oid_block + a * K + k) * 10**6 + self.seq)
            m = torch.stack([torch.ones_like(qty), side, qty, price, oid, torch.full_like(qty, tid),
                             torch.zeros_like(qty), torch.zeros_like(qty)], -1)
            ok = (qty > 0) & (side != 0)
            m[~ok] = 0
            rows.append(m)
            if k < K:
                self.live[:, a, k, 0] = torch.where(ok, oid, torch.zeros_like(oid))
                self.live[:, a, k, 1] = side
                self.live[:, a, k, 2] = price
        if market is not None:
            side, q = market[:, 0], market[:, 1]
            # a marketable order executes against the opposite side: the message carries the resting
            # side and an extreme limit (type 4: execution of visible liquidity)
            far = torch.where(side > 0, torch.full_like(q, 10**9), torch.ones_like(q))
            oid = torch.full_like(q, AGENT_OID_BASE + (oid_block + 90 + a) * 10**6 + self.seq)
            m = torch.stack([torch.full_like(q, 4), -side, q, far, oid, torch.full_like(q, tid),
                             torch.zeros_like(q), torch.zeros_like(q)], -1)
            m[(q <= 0) | (side == 0)] = 0
            rows.append(m)
        return rows

    def _state(self, inv: torch.Tensor) -> Dict[str, torch.Tensor]:
        from .agents import touch
        bb, ba, mid = touch(self.engine.l2(1).long().cpu(), self.tick)
        return {"best_bid": bb, "best_ask": ba, "mid": mid, "inventory": inv, "time_left": self.time_left()}


class MarketMakingEnv(_Quoting, BaseLOBEnv):
    """One (or several) market makers.  ``action_space`` and ``reward_function`` select one
    of the builders / rewards of ``envs/agents.py`` (the reference's config strings); the
    default quotes one bid and one ask at mid -/+ an offset and is rewarded with the change
    of mark-to-market PnL minus ``inventory_penalty`` per share held."""

    OFFSETS = (1, 2, 3, 5, 8)

    OBS_SPACES = ("basic", "engineered", "features", "messages")

    def __init__(self, *a, quote_size: int = 100, inventory_penalty: float = 0.01, n_mm: int = 1,
                 action_space: str = "offsets", reward_function: str = "pnl_inventory", inv_penalty: str = "linear",
                 reference_price: str = "mid", eta: float = 0.5, gamma: float = 1.0, lam: float = 0.0,
                 rebate_bps: float = 0.0, n_levels: int = 3, avst_k: float = 1.5, avst_var: float = 2.0,
                 inv_threshold: float = 10.0, unwind_price: str = "none", unwind_penalty: int = 0,
                 clip_reward: bool = False, volume_bonus: str = "none", exclude_extreme_spreads: bool = False,
                 auto_liquidate_threshold: int = 0, auto_liquidate_alpha: float = 1.0,
                 observation_space: str = "features", normalize: bool = True, **kw):
        from .agents import INV_PENALTIES, MM_ACTION_SPACES, MM_REWARDS, UNWIND_PRICES
        super().__init__(*a, n_agents=n_mm, **kw)
        if action_space not in MM_ACTION_SPACES or reward_function not in MM_REWARDS:
            raise ValueError(f"action_space in {MM_ACTION_SPACES}, reward_function in {MM_REWARDS}")
        if inv_penalty not in INV_PENALTIES or unwind_price not in UNWIND_PRICES:
            raise ValueError(f"inv_penalty in {INV_PENALTIES}, unwind_price in {UNWIND_PRICES}")
        if volume_bonus not in ("none", "market_share") or observation_space not in self.OBS_SPACES:
            raise ValueError(f"volume_bonus in ('none', 'market_share'), observation_space in {self.OBS_SPACES}")
        self.size, self.pen, self.n_mm = quote_size, inventory_penalty, n_mm
        self.tids = [1000 + i for i in range(n_mm)]
        self.space, self.reward_fn, self.inv_pen_kind = action_space, reward_function, inv_penalty
        self.ref_price, self.eta, self.gamma, self.lam, self.rebate = reference_price, eta, gamma, lam, rebate_bps
        self.n_levels, self.avst_k, self.avst_var = n_levels, avst_k, avst_var
        # reward shaping and episode-end options of the reference's market-making config
        # (jaxob_config.py MarketMaking_EnvironmentConfig; mm_env.py:2206-2246 the unwind,
        # :2435-2473 penalties, clipping, the market-share bonus, extreme spreads)
        self.inv_threshold, self.unwind, self.unwind_pen = inv_threshold, unwind_price, unwind_penalty
        self.clip, self.vol_bonus, self.no_extreme = clip_reward, volume_bonus, exclude_extreme_spreads
        # auto-liquidation (mm_env.py:1086-1094): above |inventory| > threshold the quotes are replaced
        # by an immediate-or-cancel order of alpha x inventory against the position
        self.liq_thr, self.liq_alpha = auto_liquidate_threshold, auto_liquidate_alpha
        self.obs_space, self.normalize = observation_space, normalize

    # the reference's MarketMaking_EnvironmentConfig field -> keyword here
    # (src/matching_engine/jaxob/jaxob_config.py:58-130)
    REFERENCE_CONFIG = {
        "action_space": "action_space", "reward_function": "reward_function", "inv_penalty": "inv_penalty",
        "inv_penalty_lambda": "inventory_penalty", "inv_penalty_threshold": "inv_threshold",
        "reference_price": "reference_price", "unwind_price": "unwind_price",
        "unwind_price_penalty": "unwind_penalty", "clip_reward": "clip_reward",
        "volume_traded_bonus": "volume_bonus", "exclude_extreme_spreads": "exclude_extreme_spreads",
        "auto_liquidate_threshold": "auto_liquidate_threshold", "auto_liquidate_alpha": "auto_liquidate_alpha",
        "observation_space": "observation_space", "normalize": "normalize", "inventoryPnL_eta": "eta",
        "inventoryPnL_gamma": "gamma", "unrealizedPnL_lambda": "lam", "rebate_bps": "rebate_bps",
        "avst_k_parameter": "avst_k", "avst_var_parameter": "avst_var", "fixed_quant_value": "quote_size",
    }

    @classmethod
    def from_reference_config(cls, windows, n_envs: int, cfg: Dict, **kw):
        """Build from the reference's market-making config (a dict of its field names).  Fields
        without a counterpart here (debug and plotting switches, ``time_delay_obs_act``, the
        message-token observation spaces) are returned unused in ``env.unused_config``."""
        args, unused = {}, {}
        for k, v in cfg.items():
            if k in cls.REFERENCE_CONFIG:
                args[cls.REFERENCE_CONFIG[k]] = v
            else:
                unused[k] = v
        if args.get("reference_price") == "best_bid_ask":
            args["reference_price"] = "far_touch"
        if args.get("observation_space") not in (None,) + cls.OBS_SPACES:
            unused["observation_space"] = args.pop("observation_space")
        args.update(kw)
        env = cls(windows, n_envs, **args)
        env.unused_config = unused
        return env

    def reset(self, idx=None):
        obs = super().reset(idx)
        z = lambda: torch.zeros(self.n, self.n_mm, dtype=torch.long)
        self.inv, self.cash = z(), z().double()
        self._init_live(self.n_mm, 2 * self.n_levels if self.space == "fixed_prices" else 2)
        self.pnl_prev = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        self.pv_prev = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        return self._obs(obs)

    def _obs(self, o):
        o = dict(o)
        o["inventory"] = self.inv.clone()
        return o

    def action_messages(self, actions: torch.Tensor, mid: Optional[torch.Tensor] = None) -> torch.Tensor:
        """actions (n, n_mm[, d]) -> (n, m, 8) messages: every market maker's cancels, new
        orders and marketable orders."""
        from .agents import mm_orders
        rows = []
        for a in range(self.n_mm):
            inv = self.inv[:, a]
            st = self._state(inv)
            if mid is not None:
                st["mid"] = mid
            orders, market = mm_orders(self.space, actions[:, a], st, self.size, self.tick, self.n_levels,
                                       self.avst_k, self.avst_var)
            if self.space != "directional_trading":
                market = torch.zeros(self.n, 2, dtype=torch.long) if self.liq_thr > 0 else None
            if self.liq_thr > 0:
                liq = inv.abs() > self.liq_thr
                qty = (self.liq_alpha * inv.abs().double()).round().long()
                orders = torch.where(liq[:, None, None], torch.zeros_like(orders), orders)
                market = torch.where(liq[:, None], torch.stack([-inv.sign(), qty], -1), market)
            rows += self._order_messages(a, self.tids[a], orders, market)
        return torch.stack(rows, 1)

    def agent_observation(self, obs: Dict[str, torch.Tensor]) -> torch.Tensor:
        """(n, n_mm, d) observation vectors of the market makers (``observation_space``):
        ``basic`` the inventory, ``engineered`` the inventory and the spread (price units),
        each as (x - mean) / scale with the reference's constants when ``normalize``
        (``mm_env.py:2881-2990``: inventory / 10, spread / 1e4; keys in sorted order), and
        ``features`` the book features of ``features()``, ``messages`` the step's data
        messages (engine rows, flattened)."""
        if self.obs_space == "features":
            return features(obs, self.n_mm)
        if self.obs_space == "messages":
            # the step's data messages as engine rows (the reference's raw "messages" space),
            # zeros before the first step; every market maker sees the same rows
            m = self.last_data.reshape(self.n, -1).float()
            return m[:, None].expand(-1, self.n_mm, -1).contiguous()
        inv = obs["inventory"].double()
        cols = [inv / 10.0 if self.normalize else inv]
        if self.obs_space == "engineered":
            spread = (obs["spread"] * self.tick).double()[:, None].expand(-1, self.n_mm)
            cols.append(spread / 1e4 if self.normalize else spread)
        return torch.stack(cols, -1).float()

    def _rewards(self, trades, mid0, obs, spread0=None):
        from .agents import agent_trades, inventory_penalty, mm_reward, touch, unwind_fill
        bb, ba, _ = touch(obs["l2"], self.tick)
        rew = torch.zeros(self.n, self.n_mm, dtype=torch.float64)
        valid = trades[..., 0] >= 0
        step_volume = torch.where(valid, trades[..., 1].abs(), torch.zeros_like(trades[..., 1])).sum(-1)
        self.unwound = torch.zeros(self.n, self.n_mm, dtype=torch.long)
        fin = self.ended & ~self.prev_ended              # episodes that ended with this step
        for a, tid in enumerate(self.tids):
            bq, bv, sq, sv = agent_trades(trades, tid)
            traded = bq + sq
            inv_prev = self.inv[:, a].clone()
            if self.unwind != "none" and bool(fin.any()):
                # the last step flattens what is left with one artificial fill
                u = unwind_fill(self.unwind, inv_prev + bq - sq, mid0, obs["mid"], bb, ba, self.tick, self.unwind_pen)
                ubq, ubv, usq, usv = (torch.where(fin, x, torch.zeros_like(x)) for x in u)
                bq, bv, sq, sv = bq + ubq, bv + ubv, sq + usq, sv + usv
                self.unwound[:, a] = usq - ubq
            self.inv[:, a] += bq - sq
            self.cash[:, a] += (sv - bv).double()
            if self.reward_fn == "pnl_inventory":
                pnl = self.cash[:, a] + self.inv[:, a].double() * obs["mid"].double()
                r = (pnl - self.pnl_prev[:, a]) / self.tick - self.pen * self.inv[:, a].double().abs()
                self.pnl_prev[:, a] = pnl
            else:
                r, pv = mm_reward(self.reward_fn, buy_q=bq, buy_v=bv, sell_q=sq, sell_v=sv, inv_prev=inv_prev,
                                  inv=self.inv[:, a], cash=self.cash[:, a], mid0=mid0, mid1=obs["mid"], best_bid=bb,
                                  best_ask=ba, tick=self.tick, reference_price=self.ref_price, eta=self.eta,
                                  gamma=self.gamma, lam=self.lam, rebate_bps=self.rebate, pv_prev=self.pv_prev[:, a])
                self.pv_prev[:, a] = pv
                r = r + inventory_penalty(self.inv_pen_kind, self.inv[:, a], self.pen, self.size, self.inv_threshold)
            if self.clip:
                r = r.clamp(-10000.0, 10000.0)
            if self.vol_bonus == "market_share":
                share = traded.double() / step_volume.clamp(min=1).double()
                r = r + r.abs() * share
            if self.no_extreme:
                # no reward while the spread exceeds 10% of the mid (before or after the step)
                wide = (obs["spread"] * self.tick).double() > 0.1 * obs["mid"].double()
                if spread0 is not None:
                    wide |= (spread0 * self.tick).double() > 0.1 * mid0.double()
                r = torch.where(wide, torch.zeros_like(r), r)
            rew[:, a] = r
        rew[self.prev_ended] = 0.0                       # frozen episodes earn nothing
        return rew

    def step(self, actions: torch.Tensor):
        obs0 = self.observe()
        trades, _ = self.step_messages(self.action_messages(actions, obs0["mid"]))
        obs = self.observe()
        rew = self._rewards(trades, obs0["mid"], obs, obs0["spread"])   # updates inventory and cash first
        return self._obs(obs), rew, self.done


class ExecutionEnv(_Quoting, BaseLOBEnv):
    """Buy or sell ``target`` shares before the episode ends (``task``: ``buy``, ``sell`` or
    ``random`` -- a side drawn per environment at every reset; default from ``side``, 1 buy
    / 0 sell).  ``action_space`` / ``reward_function`` pick an execution builder / reward of
    ``envs/agents.py``; the default sends a marketable child order of a size from a table
    and is rewarded with the negative shortfall against the arrival mid.  At the last step
    (``end_fn``) either a marketable order sweeps what is left (``sweep``), or the rest is
    booked as one artificial fill at the reference price moved ``doom_price_penalty`` ticks
    against the agent (``unwind``: the step's average mid or the far touch, as the
    reference's ``exec_env.py:1519-1560``).  ``self.info`` holds the step's statistics
    (shares left, the unwound quantity, the other traders' VWAP, advantage, drift and their
    running means over the episode)."""

    SIZES = (0, 50, 100, 200, 400)

    def __init__(self, *a, target: int = 1000, side: int = 1, action_space: str = "sizes",
                 reward_function: str = "slippage", clip: int = 100, lam: float = 1.0, task: Optional[str] = None,
                 end_fn: str = "sweep", reference_price: str = "mid", doom_price_penalty: int = 5,
                 reward_scaling: float = 1.0, **kw):
        from .agents import EXEC_ACTION_SPACES, EXEC_REWARDS
        super().__init__(*a, n_agents=1, **kw)
        if action_space not in EXEC_ACTION_SPACES or reward_function not in EXEC_REWARDS:
            raise ValueError(f"action_space in {EXEC_ACTION_SPACES}, reward_function in {EXEC_REWARDS}")
        task = task or ("buy" if side == 1 else "sell")
        if task not in ("buy", "sell", "random") or end_fn not in ("sweep", "unwind") or \
                reference_price not in ("mid", "far_touch"):
            raise ValueError("task in (buy, sell, random), end_fn in (sweep, unwind), reference_price in (mid, far_touch)")
        self.target, self.side, self.tid, self.task = target, side, 2000, task
        self.space, self.reward_fn, self.clip, self.lam = action_space, reward_function, clip, lam
        self.end_fn, self.ref_price, self.doom_pen, self.scaling = end_fn, reference_price, doom_price_penalty, \
            reward_scaling

    def reset(self, idx=None):
        o = super().reset(idx)
        if self.task == "random":
            self.sell = torch.from_numpy(self.rng.integers(0, 2, size=self.n).astype(bool))
        else:
            self.sell = torch.full((self.n,), self.task == "sell", dtype=torch.bool)
        self.done_qty = torch.zeros(self.n, dtype=torch.long)
        self.cash = torch.zeros(self.n, dtype=torch.float64)
        self.arrival = o["mid"].clone()
        self._init_live(1, 3)
        z = lambda: torch.zeros(self.n, dtype=torch.float64)
        self.info = {"vwap_rm": z(), "slippage_rm": z(), "advantage_rm": z(), "drift_rm": z()}
        o["remaining"] = torch.full((self.n,), self.target)
        o["is_sell"] = self.sell.clone()
        return o

    def step(self, actions: torch.Tensor):
        """actions: (n,) indices, or (n, 4) sizes for ``fixed_prices``."""
        from .agents import agent_trades, exec_orders, exec_reward, touch
        sell = self.sell
        rem = (self.target - self.done_qty).clamp(min=0)
        st = self._state(self.done_qty)
        orders, take = exec_orders(self.space, actions, st, rem, self.clip, self.steps_left(), sell, self.tick)
        last = self.last_step()
        if self.end_fn == "sweep":
            take = torch.where(last, rem, take)           # the last step sweeps what is left
            orders = torch.where(last[:, None, None], torch.zeros_like(orders), orders)
        sgn = torch.where(sell, -1, 1)
        market = torch.stack([sgn * (take > 0), take], -1)
        mid0 = st["mid"]
        trades, _ = self.step_messages(torch.stack(self._order_messages(0, self.tid, orders, market, 50), 1))
        bq, bv, sq, sv = agent_trades(trades, self.tid)
        filled, value = torch.where(sell, sq, bq), torch.where(sell, sv, bv)
        o = self.observe()
        bb, ba, _ = touch(o["l2"], self.tick)
        mid_avg = (mid0 + o["mid"]) // 2
        unwound = torch.zeros_like(filled)
        if self.end_fn == "unwind" and bool(last.any()):
            left = torch.where(last, (rem - filled).clamp(min=0), torch.zeros_like(filled))
            pen = self.doom_pen * self.tick
            if self.ref_price == "mid":
                px = torch.where(sell, mid_avg - pen, mid_avg + pen)
            else:
                px = torch.where(sell, bb - pen, ba + pen)
            px = px // self.tick * self.tick
            unwound = left
            filled, value = filled + left, value + left * px
        self.done_qty += filled
        self.cash += torch.where(sell, value, -value).double()
        # the rest of the market in this step (its VWAP for the vwap rewards)
        valid = trades[..., 0] >= 0
        mine = (trades[..., 6] == self.tid) | (trades[..., 7] == self.tid)
        other = valid & ~mine
        oq = torch.where(other, trades[..., 1].abs(), torch.zeros_like(trades[..., 1])).long()
        mq, mv = oq.sum(-1), (oq * trades[..., 0].long()).sum(-1)
        left = (self.target - self.done_qty).clamp(min=0)
        rew = exec_reward(self.reward_fn, filled=filled, value=value, market_q=mq, market_v=mv,
                          arrival=self.arrival, target=self.target, sell=sell, tick=self.tick, lam=self.lam,
                          remaining=left, mid_avg=mid_avg, scaling=self.scaling)
        live = ~self.prev_ended
        rew = torch.where(live, rew, torch.zeros_like(rew))
        # step statistics and their running means (exec_env.py:1700-1760)
        d = torch.float64
        sg = torch.where(sell, 1.0, -1.0).to(d)
        vwap = torch.where(mq > 0, mv.to(d) / mq.clamp(min=1).to(d), mid_avg.to(d)) / self.tick
        adv = sg * (value.to(d) / self.tick - vwap * filled.to(d))
        drift = sg * filled.to(d) * (vwap - self.arrival.to(d) / self.tick)
        k = torch.minimum(torch.full_like(self.steps_env, self.t), self.steps_env).clamp(min=1).to(d)
        for key, v in (("vwap_rm", vwap), ("advantage_rm", adv), ("drift_rm", drift), ("slippage_rm", adv + drift)):
            self.info[key] = torch.where(live, self.info[key] + (v - self.info[key]) / k, self.info[key])
        self.info.update(quant_left=left, doom_quant=unwound, p_vwap=vwap, advantage=adv, drift=drift)
        o["remaining"] = self.target - self.done_qty
        o["is_sell"] = sell.clone()
        return o, rew, self.done


class MultiAgentEnv(MarketMakingEnv):
    """Market makers and executors trading on the same books -- the reference's multi-agent
    environment (``environment/jaxen/marl_env.py:212-470``).  Every agent builds its messages
    from the book as it stands before the step; the step then applies all agents' cancels,
    then their new orders (in a random order per environment and step with
    ``shuffle_action_messages``), then the step's data messages.  Rewards are
    (n, n_mm + n_exec): the market makers' (the ``MarketMakingEnv`` options) followed by the
    executors' (the ``ExecutionEnv`` action spaces and rewards, ``exec_*`` keywords; the last
    step sweeps what an executor has left).  ``exec_qty`` keeps the plain interface: a
    marketable sell of that many shares by a trader outside the agents."""

    def __init__(self, *a, n_mm: int = 2, n_exec: int = 0, exec_target: int = 1000, exec_task: str = "sell",
                 exec_action_space: str = "sizes", exec_reward: str = "slippage", exec_clip: int = 100,
                 exec_lam: float = 1.0, shuffle_action_messages: bool = False, **kw):
        from .agents import EXEC_ACTION_SPACES, EXEC_REWARDS
        super().__init__(*a, n_mm=n_mm, **kw)
        if exec_action_space not in EXEC_ACTION_SPACES or exec_reward not in EXEC_REWARDS or \
                exec_task not in ("buy", "sell", "random"):
            raise ValueError(f"exec_action_space in {EXEC_ACTION_SPACES}, exec_reward in {EXEC_REWARDS}, "
                             f"exec_task in (buy, sell, random)")
        self.n_exec, self.exec_target, self.exec_task = n_exec, exec_target, exec_task
        self.exec_space, self.exec_reward_fn, self.exec_clip, self.exec_lam = exec_action_space, exec_reward, \
            exec_clip, exec_lam
        self.exec_tids = [2000 + i for i in range(n_exec)]
        self.exec_tid = 2000 + n_exec                 # the plain ``exec_qty`` seller
        self.shuffle = shuffle_action_messages
        self.n_agents = n_mm + n_exec

    def reset(self, idx=None):
        obs = super().reset(idx)
        self._init_live(self.n_mm + self.n_exec, max(self.live.shape[2], 3))
        E = self.n_exec
        if self.exec_task == "random":
            self.exec_sell = torch.from_numpy(self.rng.integers(0, 2, size=(self.n, E)).astype(bool))
        else:
            self.exec_sell = torch.full((self.n, E), self.exec_task == "sell", dtype=torch.bool)
        self.exec_done = torch.zeros(self.n, E, dtype=torch.long)
        self.exec_cash = torch.zeros(self.n, E, dtype=torch.float64)
        self.exec_arrival = obs["mid"].clone()
        return self._obs(obs)

    def _obs(self, o):
        o = super()._obs(o)
        if hasattr(self, "exec_done"):
            o["exec_remaining"] = self.exec_target - self.exec_done
        return o

    def _exec_messages(self, exec_actions: torch.Tensor) -> List[torch.Tensor]:
        from .agents import exec_orders
        rows = []
        last = self.last_step()
        for e in range(self.n_exec):
            rem = (self.exec_target - self.exec_done[:, e]).clamp(min=0)
            st = self._state(self.exec_done[:, e])
            sell = self.exec_sell[:, e]
            orders, take = exec_orders(self.exec_space, exec_actions[:, e], st, rem, self.exec_clip,
                                       self.steps_left(), sell, self.tick)
            take = torch.where(last, rem, take)            # the last step sweeps what is left
            orders = torch.where(last[:, None, None], torch.zeros_like(orders), orders)
            market = torch.stack([torch.where(sell, -1, 1) * (take > 0), take], -1)
            rows += self._order_messages(self.n_mm + e, self.exec_tids[e], orders, market)
        return rows

    def _order(self, msgs: torch.Tensor) -> torch.Tensor:
        """Cancels first, then the new orders (shuffled per environment if asked)."""
        typ = msgs[..., 0]
        key = torch.where(typ == 3, 0.0, 1.0).double()
        if self.shuffle:
            noise = torch.from_numpy(self.rng.random(size=tuple(typ.shape)))
            key = key + torch.where(typ == 3, 0.0, 1.0).double() * noise
        perm = torch.sort(key, dim=1, stable=True).indices
        return torch.gather(msgs, 1, perm[..., None].expand_as(msgs))

    def step(self, actions: torch.Tensor, exec_actions: Optional[torch.Tensor] = None,
             exec_qty: Optional[torch.Tensor] = None):
        """actions (n, n_mm[, d]) market-maker actions; exec_actions (n, n_exec[, d]) executor
        actions; exec_qty (n,) shares the plain outside seller sends."""
        from .agents import agent_trades, exec_reward
        obs0 = self.observe()
        msgs = self.action_messages(actions, obs0["mid"])
        if self.n_exec:
            if exec_actions is None:
                raise ValueError("exec_actions (n, n_exec) are needed with n_exec > 0")
            msgs = torch.cat([msgs, torch.stack(self._exec_messages(exec_actions), 1)], 1)
        if exec_qty is not None:
            q = exec_qty.long()
            m = torch.stack([torch.full_like(q, 4), torch.full_like(q, -1), q, torch.full_like(q, 10**9),
                             torch.full_like(q, AGENT_OID_BASE + 60 * 10**6 + self.t), torch.full_like(q, self.exec_tid),
                             torch.zeros_like(q), torch.zeros_like(q)], -1)[:, None]
            m[q <= 0] = 0
            msgs = torch.cat([msgs, m], 1)
        trades, _ = self.step_messages(self._order(msgs))
        obs = self.observe()
        rew = self._rewards(trades, obs0["mid"], obs, obs0["spread"])
        if self.n_exec:
            valid = trades[..., 0] >= 0
            mine = torch.zeros_like(valid)
            for tid in self.tids + self.exec_tids:
                mine |= (trades[..., 6] == tid) | (trades[..., 7] == tid)
            oq = torch.where(valid & ~mine, trades[..., 1].abs(), torch.zeros_like(trades[..., 1])).long()
            mq, mv = oq.sum(-1), (oq * trades[..., 0].long()).sum(-1)
            er = torch.zeros(self.n, self.n_exec, dtype=torch.float64)
            for e, tid in enumerate(self.exec_tids):
                bq, bv, sq, sv = agent_trades(trades, tid)
                sell = self.exec_sell[:, e]
                filled, value = torch.where(sell, sq, bq), torch.where(sell, sv, bv)
                self.exec_done[:, e] += filled
                self.exec_cash[:, e] += torch.where(sell, value, -value).double()
                left = (self.exec_target - self.exec_done[:, e]).clamp(min=0)
                er[:, e] = exec_reward(self.exec_reward_fn, filled=filled, value=value, market_q=mq, market_v=mv,
                                       arrival=self.exec_arrival, target=self.exec_target, sell=sell,
                                       tick=self.tick, lam=self.exec_lam, remaining=left,
                                       mid_avg=(obs0["mid"] + obs["mid"]) // 2)
            er[self.prev_ended] = 0.0
            rew = torch.cat([rew, er], 1)
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
