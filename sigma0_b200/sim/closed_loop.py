"""A quoting policy against a frozen episode: decision points spread over the window's wall
clock, the background flow replayed through the engine between them, the policy's quotes
resting in the same book.

The reference's loop (``src/post_training/heuristic_learning/mm_sim.py:58-366``) fixes the
contract kept here:

* ``n_steps`` decision points evenly spaced between ``warmup_s`` after the episode's first
  message and its last one (no quoting during the warm-up: inference over a window takes
  time);
* the policy sees an observation dict (time left, touch, mid, spread in ticks, level sizes,
  inventory, cash, mark-to-market PnL, its resting quote prices, the fills since its last
  decision, the episode's signal) and answers ``{"post_bid", "post_ask", "cancel_bid",
  "cancel_ask", "size"}``; quotes sit at the touch, a quote already resting at the touch is
  kept rather than re-queued, sizes are capped at ``size_cap`` and a side is not quoted once
  the inventory reached ``inventory_cap`` in that direction;
* the trade buffer is cleared before every engine call, so a step's fills are exactly that
  step's trades;
* at the end the inventory is flattened at the final mid moved ``unwind_penalty_ticks``
  against the agent;
* a policy that raises ends the episode with an error in the trajectory instead of ending
  the caller.

``symmetric_touch`` is the baseline every candidate is compared with: both sides at the
touch, always, within the caps.  Episodes are the dicts of ``sim.frozen`` (``init_book``,
``background`` engine rows, ``signal_*`` curve entries).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import numpy as np

from ..engine.book import EMPTY, EngineConfig, OrderBook, init_msgs_from_l2

AGENT_TID = 424_242
EMPTY_ASK = 2 ** 31 - 1


@dataclass
class SimConfig:
    n_levels: int = 10
    n_steps: int = 60
    warmup_s: float = 1.0
    size_cap: int = 10
    inventory_cap: int = 50
    unwind_penalty_ticks: int = 1
    tick: int = 100


@dataclass
class StepRecord:
    t_ns: int
    mid: float
    best_bid: int
    best_ask: int
    inventory: int
    cash: float
    action: Dict[str, Any]
    fills: List[Dict[str, int]] = field(default_factory=list)


@dataclass
class Trajectory:
    steps: List[StepRecord]
    realized_pnl: float
    final_inventory: int
    unwind_pnl: float
    total_pnl: float
    n_fills: int
    error: Optional[str] = None


def observation(book: np.ndarray, t_ns: int, end_ns: int, inventory: int, cash: float, realized: float,
                my_bid: Optional[int], my_ask: Optional[int], fills: List[Dict[str, int]],
                signal: Optional[Dict[str, Any]], tick: int = 100) -> Dict[str, Any]:
    ask, bid = int(book[0]), int(book[2])
    return {"time_left_s": max(0.0, (end_ns - t_ns) / 1e9), "best_bid": bid, "best_ask": ask,
            "mid": (ask + bid) / 2.0, "spread_ticks": (ask - bid) / tick, "bid_sizes": book[3::4].tolist(),
            "ask_sizes": book[1::4].tolist(), "inventory": inventory, "cash": cash, "realized_pnl": realized,
            "my_bid_px": my_bid, "my_ask_px": my_ask, "fills_since_last": fills, "signal": signal or {}}


def symmetric_touch(obs: Dict[str, Any], state: Dict[str, Any]) -> Dict[str, Any]:
    cap = state.get("inventory_cap", 50)
    return {"post_bid": obs["inventory"] < cap, "post_ask": obs["inventory"] > -cap, "cancel_bid": True,
            "cancel_ask": True, "size": state.get("size", 10)}


def _signal(episode: Dict[str, Any]) -> Dict[str, Any]:
    return {k[len("signal_"):]: (v.tolist() if hasattr(v, "tolist") else v)
            for k, v in episode.items() if k.startswith("signal_") and k != "signal_seeds"}


def run_frozen_episode(policy_fn: Callable[[Dict, Dict], Dict], episode: Dict[str, Any], cfg: SimConfig = SimConfig(),
                       policy_state: Optional[Dict[str, Any]] = None,
                       engine: EngineConfig = EngineConfig()) -> Trajectory:
    bg = np.asarray(episode["background"], np.int64)
    init = np.asarray(episode["init_book"], np.int64)
    t_all = bg[:, 6] * 1_000_000_000 + bg[:, 7]
    t0, t_end = int(t_all[0]), int(t_all[-1])
    bounds = np.linspace(t0 + int(cfg.warmup_s * 1e9), t_end, cfg.n_steps + 1).astype(np.int64)
    ob = OrderBook(engine)
    ob.process_many(init_msgs_from_l2(init, engine, (int(bg[0, 6]), int(bg[0, 7]))))
    pstate = dict(policy_state or {})
    pstate.setdefault("size", cfg.size_cap)
    pstate.setdefault("inventory_cap", cfg.inventory_cap)
    signal = _signal(episode)
    inventory, cash, realized = 0, 0.0, 0.0
    live: Dict[int, Dict[str, int]] = {}            # our resting orders by id: side, price, remaining qty
    my_bid = my_ask = None
    next_oid = -1000
    steps: List[StepRecord] = []
    cursor = int(np.searchsorted(t_all, bounds[0], side="left"))

    def push(msgs: np.ndarray):
        ob.trades[:] = EMPTY                         # this call's trades only
        ob.process_many(msgs)
        return ob.trades.copy()

    if cursor:
        push(bg[:cursor])
    for k in range(cfg.n_steps):
        lo, hi = int(bounds[k]), int(bounds[k + 1])
        book = ob.l2(cfg.n_levels)
        ask, bid = int(book[0]), int(book[2])
        if bid <= 0 or ask <= 0 or ask >= EMPTY_ASK:
            continue
        ts, tns = lo // 1_000_000_000, lo % 1_000_000_000
        obs = observation(book, lo, t_end, inventory, cash, realized, live.get(my_bid, {}).get("px"),
                          live.get(my_ask, {}).get("px"), steps[-1].fills if steps else [], signal, cfg.tick)
        try:
            action = policy_fn(obs, pstate) or {}
        except Exception as exc:                      # a broken policy ends its episode, not the run
            return Trajectory(steps, realized, inventory, 0.0, realized, sum(len(s.fills) for s in steps),
                              error=f"policy raised at step {k}: {exc!r}")
        size = int(min(abs(int(action.get("size", 0))), cfg.size_cap))
        out: List[List[int]] = []
        want_bid = bool(action.get("post_bid")) and size > 0 and inventory < cfg.inventory_cap
        want_ask = bool(action.get("post_ask")) and size > 0 and inventory > -cfg.inventory_cap

        def cancel(oid, wanted):
            if not wanted or oid is None or oid not in live:
                return oid
            o = live.pop(oid)
            out.append([3, o["side"], 10 ** 9, o["px"], oid, AGENT_TID, ts, tns])     # delete the rest
            return None
        keep_bid = want_bid and my_bid in live and live[my_bid]["px"] == bid
        keep_ask = want_ask and my_ask in live and live[my_ask]["px"] == ask
        my_bid = cancel(my_bid, action.get("cancel_bid") and not keep_bid)
        my_ask = cancel(my_ask, action.get("cancel_ask") and not keep_ask)
        for want, side, px in ((want_bid, 1, bid), (want_ask, -1, ask)):
            if want and (my_bid if side > 0 else my_ask) is None:
                next_oid -= 1
                live[next_oid] = {"side": side, "px": px, "qty": size}
                out.append([1, side, size, px, next_oid, AGENT_TID, ts, tns])
                if side > 0:
                    my_bid = next_oid
                else:
                    my_ask = next_oid
        nxt = int(np.searchsorted(t_all, hi, side="left"))
        msgs = np.concatenate([np.asarray(out, np.int64).reshape(-1, 8), bg[cursor:nxt]])
        trades = push(msgs)
        cursor = nxt
        fills = []
        for tr in trades[trades[:, 0] != EMPTY]:
            for col in (2, 3):                           # our order resting or aggressing
                oid = int(tr[col])
                if oid in live:
                    o = live[oid]
                    q = min(abs(int(tr[1])), o["qty"])
                    fills.append({"side": o["side"], "px": int(tr[0]), "qty": q})
                    o["qty"] -= q
                    if o["qty"] <= 0:
                        del live[oid]
        my_bid = my_bid if my_bid in live else None        # a filled quote frees its side
        my_ask = my_ask if my_ask in live else None
        for f in fills:
            signed = f["qty"] if f["side"] > 0 else -f["qty"]
            inventory += signed
            cash -= signed * f["px"]
        realized = cash + inventory * (ask + bid) / 2.0
        steps.append(StepRecord(lo, (ask + bid) / 2.0, bid, ask, inventory, cash, dict(action), fills))
    fb = ob.l2(cfg.n_levels)
    fa, fbid = int(fb[0]), int(fb[2])
    mid = (fa + fbid) / 2.0 if fbid > 0 and 0 < fa < EMPTY_ASK else (steps[-1].mid if steps else 0.0)
    pen = cfg.unwind_penalty_ticks * cfg.tick
    px = mid - pen if inventory > 0 else mid + pen
    unwind = inventory * px if inventory else 0.0           # selling a long, buying back a short
    total = cash + unwind
    return Trajectory(steps, realized, inventory, total - realized, total, sum(len(s.fills) for s in steps))


def compare_to_baseline(policy_fn: Callable, episodes: List[Dict[str, Any]], cfg: SimConfig = SimConfig()) -> Dict:
    """Mean total PnL of ``policy_fn`` and of ``symmetric_touch`` over the same episodes and
    the mean per-episode difference (a ticker-independent number to optimise)."""
    ours = [run_frozen_episode(policy_fn, ep, cfg) for ep in episodes]
    base = [run_frozen_episode(symmetric_touch, ep, cfg) for ep in episodes]
    d = [a.total_pnl - b.total_pnl for a, b in zip(ours, base)]
    return {"policy_pnl": float(np.mean([t.total_pnl for t in ours])),
            "baseline_pnl": float(np.mean([t.total_pnl for t in base])), "delta_mean": float(np.mean(d)),
            "errors": [t.error for t in ours if t.error]}
