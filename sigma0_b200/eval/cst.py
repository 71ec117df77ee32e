"""Cont-Stoikov-Talreja order-book model: parameter estimation and simulation.

The reference ships the CST model as a baseline generator for LOB-Bench
(``src/lobpipeline/scorer/lob_bench/cst_model/cst.py``, ``param_estimation.py``).  The model
(Cont, Stoikov & Talreja, "A stochastic model for order book dynamics", Operations Research
2010): on a price grid of ticks, in units of one order size,

* limit buy orders arrive i ticks below the best ask (and limit sells i ticks above the
  best bid) at rate lambda(i) = k i^-alpha, i = 1..D;
* market buy and sell orders each arrive at rate mu and take one unit from the touch;
* every resting unit i ticks from the opposite best price is cancelled at rate theta(i).

``estimate`` reads the rates off a message stream (this package's message / L2 arrays) the
way the paper does: lambda(i) from the count of new limit orders at distance i per unit
time (k, alpha by a least-squares fit of log lambda on log i), mu from the executed volume
per unit time, theta(i) from the cancelled volume at distance i divided by the time-averaged
queue at that distance.  ``simulate`` runs the continuous-time Markov chain (Gillespie) and
writes messages and the 10-level book after each event, so the stream scores against real
data with ``eval/lob_bench.py`` like any generator.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Tuple

import numpy as np

LIMIT, DELETE, EXEC = 1, 3, 4


@dataclass
class CSTParams:
    k: float = 1.0
    alpha: float = 0.5
    mu: float = 1.0
    theta: np.ndarray = field(default_factory=lambda: np.full(10, 0.2))
    tick: int = 100
    unit: int = 100                 # shares per order unit

    @property
    def depth(self) -> int:
        return len(self.theta)

    def lam(self) -> np.ndarray:
        i = np.arange(1, self.depth + 1, dtype=np.float64)
        return self.k * i ** (-self.alpha)


def _t(m):
    return m[:, 0].astype(np.float64) + m[:, 1].astype(np.float64) * 1e-9


def estimate(msgs: np.ndarray, l2: np.ndarray, tick: int = 100, depth: int = 10) -> CSTParams:
    m, b = np.asarray(msgs), np.asarray(l2)
    T = max(float(_t(m)[-1] - _t(m)[0]), 1e-9)
    prev = np.vstack([b[:1], b[:-1]])
    ask, bid = prev[:, 0].astype(np.float64), prev[:, 2].astype(np.float64)
    lim = m[:, 2] == LIMIT
    unit = float(np.mean(m[lim, 4])) if lim.any() else 100.0
    # distance of each new limit order from the opposite best price
    dist = np.where(m[:, 6] > 0, (ask - m[:, 5]) / tick, (m[:, 5] - bid) / tick)
    lam = np.zeros(depth)
    for i in range(1, depth + 1):
        lam[i - 1] = np.sum(lim & (np.round(dist) == i)) / (2.0 * T)        # per side
    ok = lam > 0
    if ok.sum() >= 2:
        slope, icpt = np.polyfit(np.log(np.arange(1, depth + 1)[ok]), np.log(lam[ok]), 1)
        k, alpha = float(np.exp(icpt)), float(-slope)
    else:
        k, alpha = float(lam.max() if ok.any() else 1.0), 0.5
    ex = m[:, 2] == EXEC
    mu = float(m[ex, 4].sum() / unit / (2.0 * T))
    # time-averaged queue (units) at distance i from the opposite best, from the L2 levels
    dt = np.diff(np.concatenate([_t(m), [_t(m)[-1]]]))
    q = np.zeros(depth)
    L = b.shape[1] // 4
    for lvl in range(L):
        bp, bv = b[:, 4 * lvl + 2].astype(np.float64), b[:, 4 * lvl + 3].astype(np.float64)
        ap, av = b[:, 4 * lvl].astype(np.float64), b[:, 4 * lvl + 1].astype(np.float64)
        for p, v, ref in ((bp, bv, b[:, 0]), (ap, av, b[:, 2])):
            d = np.round(np.abs(ref - p) / tick).astype(int)
            sel = (d >= 1) & (d <= depth) & (v > 0) & (np.abs(p) < 2e9)
            np.add.at(q, d[sel] - 1, v[sel] / unit * dt[sel])
    q = q / (2.0 * T)
    canc = np.isin(m[:, 2], (2, DELETE))
    cdist = np.where(m[:, 6] > 0, (ask - m[:, 5]) / tick, (m[:, 5] - bid) / tick)
    cv = np.zeros(depth)
    for i in range(1, depth + 1):
        sel = canc & (np.round(cdist) == i)
        cv[i - 1] = m[sel, 4].sum() / unit / (2.0 * T)
    theta = np.where(q > 0, cv / np.maximum(q, 1e-12), 0.0)
    return CSTParams(k=k, alpha=alpha, mu=mu, theta=theta, tick=tick, unit=int(round(unit)))


def simulate(p: CSTParams, n_events: int, seed: int = 0, mid0: int = 10_000_000, levels: int = 10,
             init_depth: int = 5, t0: float = 34_200.0) -> Tuple[np.ndarray, np.ndarray]:
    """(messages (n, 7), books (n, 4 levels)) of ``n_events`` model events."""
    rng = np.random.default_rng(seed)
    D, tick = p.depth, p.tick
    lam = p.lam()
    # book: price (ticks) -> list of [oid, units]
    bids, asks = {}, {}
    oid = [1]

    def add(book, px, units):
        book.setdefault(px, []).append([oid[0], units])
        oid[0] += 1
        return oid[0] - 1

    c = mid0 // tick
    for i in range(1, D + 1):
        add(asks, c + i, init_depth)
        add(bids, c - i, init_depth)
    msgs = np.zeros((n_events, 7), dtype=np.int64)
    books = np.zeros((n_events, 4 * levels), dtype=np.int64)
    t = t0
    for e in range(n_events):
        ba, bb = min(asks), max(bids)
        # queue (units) at distance i from the opposite best
        qb = np.array([sum(u for _, u in bids.get(ba - i, [])) for i in range(1, D + 1)], np.float64)
        qa = np.array([sum(u for _, u in asks.get(bb + i, [])) for i in range(1, D + 1)], np.float64)
        rates = np.concatenate([lam, lam, [p.mu, p.mu], p.theta * qb, p.theta * qa])
        tot = rates.sum()
        t += rng.exponential(1.0 / tot)
        j = rng.choice(len(rates), p=rates / tot)
        sec, ns = int(t), int((t - int(t)) * 1e9)
        if j < D:                                   # limit buy i ticks below the ask
            px = ba - (j + 1)
            o = add(bids, px, 1)
            row = (LIMIT, o, p.unit, px * tick, 1)
        elif j < 2 * D:                             # limit sell i ticks above the bid
            px = bb + (j - D + 1)
            o = add(asks, px, 1)
            row = (LIMIT, o, p.unit, px * tick, -1)
        elif j < 2 * D + 2:                         # market order: one unit off the touch
            buy = j == 2 * D
            book, px = (asks, ba) if buy else (bids, bb)
            q = book[px]
            q[0][1] -= 1
            o = q[0][0]
            if q[0][1] == 0:
                q.pop(0)
            if not q:
                del book[px]
                if not book:                        # never empty a side: re-seed one tick behind
                    add(book, px + (1 if buy else -1), 1)
            row = (EXEC, o, p.unit, px * tick, -1 if buy else 1)
        else:                                       # cancel one unit i ticks from the opposite best
            jj = j - 2 * D - 2
            side_b = jj < D
            i = (jj % D) + 1
            book, px = (bids, ba - i) if side_b else (asks, bb + i)
            q = book.get(px)
            if not q or (len(book) == 1 and len(q) == 1 and q[0][1] == 1):
                row = None
            else:
                k = rng.integers(len(q))
                o = q[k][0]
                q[k][1] -= 1
                if q[k][1] == 0:
                    q.pop(k)
                if not q:
                    del book[px]
                row = (DELETE, o, p.unit, px * tick, 1 if side_b else -1)
        if row is None:
            row = (LIMIT, add(bids, bb, 1), p.unit, bb * tick, 1)
        msgs[e] = (sec, ns) + row
        a_lv = sorted(asks)[:levels]
        b_lv = sorted(bids, reverse=True)[:levels]
        for L in range(levels):
            if L < len(a_lv):
                books[e, 4 * L] = a_lv[L] * tick
                books[e, 4 * L + 1] = sum(u for _, u in asks[a_lv[L]]) * p.unit
            else:
                books[e, 4 * L] = 9_999_999_999
            if L < len(b_lv):
                books[e, 4 * L + 2] = b_lv[L] * tick
                books[e, 4 * L + 3] = sum(u for _, u in bids[b_lv[L]]) * p.unit
            else:
                books[e, 4 * L + 2] = -9_999_999_999
    return msgs, books
