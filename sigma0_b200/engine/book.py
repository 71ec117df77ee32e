"""CPU reference order book with the reference engine's semantics.

This is the oracle for the batched CUDA engine (``engine/cuda_engine.py``) and
the engine used by the synthetic order-flow generator.  It keeps the
reference's fixed-capacity array layout and its exact behaviours:

* each side is an ``(n_orders, 6)`` int32 array ``[price, qty, oid, tid, sec, ns]``
  with ``-1`` rows for empty slots; trades are ``(n_trades, 8)``
  (``src/matching_engine/jaxob/JaxOrderBookArrays.py:84-112``);
* an add writes the first empty slot; a full side first evicts every order at
  the worst price (``bid_lim``/``ask_lim``, ``:403-600``, ``check_book_fill``);
* a cancel looks up the order id, then an init order at the same price with
  enough quantity (``cancel_mode`` 1), then optionally a random order at the
  price (modes 2/3); a failed lookup lands on the LAST row, exactly as the
  reference's ``.at[-1]`` does (``:115-190``);
* type-4 (execution) messages flip side and are immediate-or-cancel under the
  default interpretation (``:601-640``, ``Type4Interpretation.IOC``);
* the message switch sends anything that is not an explicit cancel or the
  all-zero no-op to ``ask_lim`` (the reference's index arithmetic, ``:623-633``);
* L2 extraction returns ``[ask_p, ask_v, bid_p, bid_v] * n_levels`` with
  ``maxint`` / ``-maxint`` prices and zero volume for missing levels
  (``get_L2_state`` ``:1266-1300``).

Engine message rows are ``[type, side, quantity, price, order_id, trader_id,
time_s, time_ns]`` (``jaxob_constants.LOBMSGFEAT``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

MAXINT = 2_147_483_647
INITID = -2
NEGATIVE_RETURN_ID = -999_999_999
EMPTY = -1

# cancel modes
STRICT_BY_ID, INCLUDE_INITS, CANCEL_UNIFORM, CANCEL_UNIFORM_AND_LARGE = 0, 1, 2, 3
# type-4 interpretations
IOC, LIM, MKT = 0, 1, 2


@dataclass(frozen=True)
class EngineConfig:
    """Engine configuration (``src/matching_engine/jaxob/jaxob_config.py:12-45``)."""
    maxint: int = MAXINT
    init_id: int = INITID
    book_depth: int = 10
    cancel_mode: int = INCLUDE_INITS
    type_4_interpretation: int = IOC
    seed: int = 42
    n_trades: int = 100
    n_orders: int = 100
    check_book_fill: bool = True

    def __post_init__(self):
        lo = self.init_id - (2 * self.book_depth - 1)
        if lo <= NEGATIVE_RETURN_ID <= self.init_id:
            raise ValueError("book_depth so deep that the miss sentinel is a valid init id")


class OrderBook:
    """One book.  ``process`` applies a single engine message in place."""

    def __init__(self, cfg: EngineConfig = EngineConfig(), seed: Optional[int] = None):
        self.cfg = cfg
        self.rng = np.random.default_rng(cfg.seed if seed is None else seed)
        self.reset()

    # -- state ----------------------------------------------------------------
    def reset(self):
        c = self.cfg
        self.asks = np.full((c.n_orders, 6), EMPTY, dtype=np.int64)
        self.bids = np.full((c.n_orders, 6), EMPTY, dtype=np.int64)
        self.trades = np.full((c.n_trades, 8), EMPTY, dtype=np.int64)

    def copy(self) -> "OrderBook":
        ob = OrderBook.__new__(OrderBook)
        ob.cfg, ob.rng = self.cfg, self.rng
        ob.asks, ob.bids, ob.trades = self.asks.copy(), self.bids.copy(), self.trades.copy()
        return ob

    # -- primitives -------------------------------------------------------------
    @staticmethod
    def _remove_nonpositive(side):
        dead = side[:, 1] <= 0
        side[dead] = EMPTY

    def _add(self, side, price, qty, oid, tid, sec, ns):
        # the reference takes the first row holding -1 in any column
        empty = np.nonzero((side == EMPTY).any(axis=1))[0]
        idx = empty[0] if len(empty) else -1
        side[idx] = [price, max(0, qty), oid, tid, sec, ns]
        self._remove_nonpositive(side)

    def _top_bid(self, side) -> int:
        maxp = side[:, 0].max()
        times = np.where(side[:, 0] == maxp, side[:, 4], self.cfg.maxint)
        tmin = times.min()
        tns = np.where(times == tmin, side[:, 5], self.cfg.maxint)
        nsmin = tns.min()
        hit = np.nonzero(tns == nsmin)[0]
        return int(hit[0]) if len(hit) else -1

    def _top_ask(self, side) -> int:
        prices = np.where(side[:, 0] == EMPTY, self.cfg.maxint, side[:, 0])
        minp = prices.min()
        times = np.where(side[:, 0] == minp, side[:, 4], self.cfg.maxint)
        tmin = times.min()
        tns = np.where(times == tmin, side[:, 5], self.cfg.maxint)
        nsmin = tns.min()
        hit = np.nonzero(tns == nsmin)[0]
        return int(hit[0]) if len(hit) else -1

    def _match_one(self, side, top, qtm, agr_oid, sec, ns, agr_tid, s):
        newq = max(0, side[top, 1] - qtm)
        qtm = int(qtm - side[top, 1])
        tr = np.nonzero(self.trades[:, 4] == EMPTY)[0]   # the reference tests column 4
        ti = tr[0] if len(tr) else -1
        self.trades[ti] = [side[top, 0], -s * (side[top, 1] - newq), side[top, 2],
                           agr_oid, sec, ns, side[top, 3], agr_tid]
        side[top, 1] = newq
        self._remove_nonpositive(side)
        return qtm

    def _match_against(self, side, is_bid_side, qtm, price, oid, sec, ns, tid, s):
        top = self._top_bid(side) if is_bid_side else self._top_ask(side)
        while True:
            p = side[top, 0]
            crosses = (p >= price) if is_bid_side else (p <= price)
            if not (crosses and qtm > 0 and p != EMPTY):
                break
            qtm = self._match_one(side, top, qtm, oid, sec, ns, tid, s)
            top = self._top_bid(side) if is_bid_side else self._top_ask(side)
        return qtm

    def _evict_if_full(self, side, worst_is_min: bool):
        if np.all(side[:, 0] >= 0):
            worst = side[:, 0].min() if worst_is_min else side[:, 0].max()
            side[side[:, 0] == worst] = EMPTY

    def _cancel_idx(self, side, price, qty, oid) -> int:
        hit = np.nonzero(side[:, 2] == oid)[0]
        if len(hit):
            return int(hit[0])
        c = self.cfg
        if c.cancel_mode == STRICT_BY_ID:
            return -1
        m = ((side[:, 0] == price) & (side[:, 2] <= c.init_id)
             & (side[:, 2] >= c.init_id - c.book_depth * 2) & (side[:, 1] >= qty))
        hit = np.nonzero(m)[0]
        if len(hit):
            return int(hit[0])
        if c.cancel_mode in (CANCEL_UNIFORM, CANCEL_UNIFORM_AND_LARGE):
            for require_qty in ((True, False) if c.cancel_mode == CANCEL_UNIFORM_AND_LARGE else (True,)):
                m = side[:, 0] == price
                if require_qty:
                    m &= side[:, 1] >= qty
                ids = np.where(m, side[:, 2], 0)
                cand = np.nonzero(ids != 0)[0]
                if len(cand):
                    pick = ids[cand[self.rng.integers(len(cand))]]
                    return int(np.nonzero(side[:, 2] == pick)[0][0])
        return -1

    def _cancel(self, side, price, qty, oid):
        idx = self._cancel_idx(side, price, qty, oid)
        side[idx, 1] = side[idx, 1] - qty          # idx == -1 -> last row, as in the reference
        self._remove_nonpositive(side)

    # -- message switch -----------------------------------------------------------
    def process(self, msg) -> None:
        t, side_raw, q, p, oid, tid, sec, ns = (int(v) for v in msg[:8])
        s = -side_raw if t == 4 else side_raw
        c = self.cfg
        if s == 0 and t == 0:
            return
        if s == -1 and t in (2, 3):
            self._cancel(self.asks, p, q, oid)
        elif s == 1 and t in (2, 3):
            self._cancel(self.bids, p, q, oid)
        elif s == 1 and t in (1, 4):
            self._limit(True, t, p, q, oid, tid, sec, ns, s)
        else:  # every other combination routes to ask_lim, like the reference switch
            self._limit(False, t, p, q, oid, tid, sec, ns, s)

    def _limit(self, is_bid, t, p, q, oid, tid, sec, ns, s):
        c = self.cfg
        if is_bid:
            rem = self._match_against(self.asks, False, q, p, oid, sec, ns, tid, s)
            if c.type_4_interpretation == MKT:
                p = c.maxint
            own = self.bids
            worst_is_min = True
        else:
            if c.type_4_interpretation == MKT:
                p = 0
            rem = self._match_against(self.bids, True, q, p, oid, sec, ns, tid, s)
            own = self.asks
            worst_is_min = False
        if c.check_book_fill:
            self._evict_if_full(own, worst_is_min)
        before = own.copy()
        self._add(own, p, rem, oid, tid, sec, ns)
        if c.type_4_interpretation in (IOC, MKT) and t == 4:
            own[:] = before   # IOC/MKT executions never rest (post-eviction, pre-add side kept)

    def process_many(self, msgs) -> None:
        for m in np.asarray(msgs):
            self.process(m)

    # -- queries ----------------------------------------------------------------------
    def l2(self, n_levels: Optional[int] = None) -> np.ndarray:
        n = n_levels or self.cfg.book_depth
        c = self.cfg
        bp = self.bids[:, 0]
        bid_prices = -np.unique(-bp)
        bid_prices = np.concatenate([bid_prices, np.full(max(0, n - len(bid_prices)), -1)])[:n]
        ap = np.where(self.asks[:, 0] == EMPTY, c.maxint, self.asks[:, 0])
        ask_prices = np.unique(ap)
        ask_prices = np.concatenate([ask_prices, np.full(max(0, n - len(ask_prices)), -1)])[:n]
        ask_prices = np.where(ask_prices == -1, c.maxint, ask_prices)
        bid_prices = np.where(bid_prices == -1, -c.maxint, bid_prices)
        bv = np.array([self.bids[self.bids[:, 0] == x, 1].sum() for x in bid_prices])
        av = np.array([self.asks[self.asks[:, 0] == x, 1].sum() for x in ask_prices])
        bv = np.maximum(bv, 0)
        av = np.maximum(av, 0)
        out = np.stack([ask_prices, av, bid_prices, bv], axis=1).reshape(-1)
        return out.astype(np.int64)

    def best_bid_ask(self):
        bi, ai = self._top_bid(self.bids), self._top_ask(self.asks)
        return self.bids[bi].copy(), self.asks[ai].copy()

    def mid_price(self) -> float:
        b, a = self.best_bid_ask()
        return (b[0] + a[0]) / 2.0


def init_msgs_from_l2(l2: np.ndarray, cfg: EngineConfig = EngineConfig(), time=(34200, 0)) -> np.ndarray:
    """Limit orders that rebuild a book from one L2 row (``init_msgs_from_l2`` ``:1045``).

    Row k of the L2 pairs (``[ask_p, ask_v, bid_p, bid_v, ...]`` reshaped to
    ``(2*levels, 2)``) becomes a limit order on the ask side for even k and the
    bid side for odd k, with ids ``init_id - k`` and trader id ``init_id``.
    """
    l2 = np.asarray(l2, dtype=np.int64)
    levels = l2.shape[0] // 4
    data = l2.reshape(levels * 2, 2)
    out = np.zeros((levels * 2, 8), dtype=np.int64)
    out[:, 3] = data[:, 0]
    out[:, 2] = data[:, 1]
    out[:, 0] = 1
    out[0::2, 1] = -1
    out[1::2, 1] = 1
    out[:, 4] = cfg.init_id - np.arange(levels * 2)
    out[:, 5] = cfg.init_id
    out[:, 6] = time[0]
    out[:, 7] = time[1]
    return out


def book_from_l2(l2: np.ndarray, cfg: EngineConfig = EngineConfig(), time=(34200, 0)) -> OrderBook:
    """Reset a book and replay the init messages of one L2 snapshot (``jorderbook.py:41``)."""
    ob = OrderBook(cfg)
    msgs = init_msgs_from_l2(l2, cfg, time)
    for m in msgs:
        ob.process(m)
    return ob
