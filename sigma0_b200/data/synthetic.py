"""Seeded synthetic order flow with book states from the matching engine.

There is no network and no LOBSTER data on the build or GPU machines, so every
benchmark and test uses this generator.  The distributions are the ones the
benchmark configurations name:

* event type in {submit 1, cancel 2, delete 3, execute 4} with p = (0.5, 0.25, 0.15, 0.10);
* side +-1 uniform;
* submit price = latent mid + discretised Laplace tick offset (scale 5, clipped +-500),
  the latent mid doing a +-1 tick random walk per message;
* size = round(lognormal(mu=4, sigma=1)) + 1;
* inter-arrival time ~ Exp(mean 1 ms), in nanoseconds.

Cancels and deletes pick a random resting order of the chosen side; executions
hit the best resting order of the chosen side (LOBSTER convention: the
direction of an execution is the side of the resting order).  When the chosen
side is empty the message becomes a submit.  Every message is replayed through
:class:`~sigma0_b200.engine.book.OrderBook`, which yields the L2 book states.

Outputs follow the reference's preprocessed layouts: 14-column message rows
(``encoding_22tok.py:391-470`` ``preproc``) and book rows
``[delta_mid, time_s, time_ns, L2...]`` holding the state BEFORE each message.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import numpy as np

from ..encoding.tokenizer import NA_VAL
from ..engine.book import EngineConfig, OrderBook, book_from_l2, MAXINT

TICK = 100
EVENT_P = (0.5, 0.25, 0.15, 0.10)


@dataclass
class SyntheticDay:
    msgs: np.ndarray          # (n, 14) preprocessed message rows
    books: np.ndarray         # (n, 3 + 4*levels) book state before each message
    engine_msgs: np.ndarray   # (n, 8) engine message rows
    l2_init: np.ndarray       # (4*levels,) book the day started from


def _initial_l2(rng, mid_ticks: int, levels: int) -> np.ndarray:
    rows = []
    for k in range(levels):
        rows += [(mid_ticks + 1 + k) * TICK, int(rng.lognormal(4, 1)) + 1,
                 (mid_ticks - 1 - k) * TICK, int(rng.lognormal(4, 1)) + 1]
    return np.array(rows, dtype=np.int64)


def _mid_from_l2(l2: np.ndarray, fallback: float) -> float:
    ap, bp = l2[0], l2[2]
    if abs(ap) >= MAXINT or abs(bp) >= MAXINT:
        return fallback
    return (ap + bp) / 2.0


def generate_day(n_msgs: int, seed: int = 0, levels: int = 10,
                 mid0_ticks: int = 10_000, cfg: EngineConfig = EngineConfig()) -> SyntheticDay:
    rng = np.random.default_rng(seed)
    l2_0 = _initial_l2(rng, mid0_ticks, levels)
    ob = book_from_l2(l2_0, cfg, (34200, 0))
    mid = mid0_ticks
    t_ns_total = 34200 * 10**9
    next_oid = 1
    # order id -> (rel price at submit, size, time_s, time_ns)
    submitted: Dict[int, Tuple[int, int, int, int]] = {}

    msgs = np.zeros((n_msgs, 14), dtype=np.int64)
    books = np.zeros((n_msgs, 3 + 4 * levels), dtype=np.float64)
    emsgs = np.zeros((n_msgs, 8), dtype=np.int64)
    prev_l2 = ob.l2(levels)
    prev_mid = _mid_from_l2(prev_l2, mid * TICK)
    for i in range(n_msgs):
        dt = int(rng.exponential(1e6))
        t_ns_total += dt
        ts, tns = divmod(t_ns_total, 10**9)
        mid += int(rng.choice((-1, 1)))
        et = int(rng.choice(4, p=EVENT_P)) + 1
        side = int(rng.choice((-1, 1)))
        size = int(round(rng.lognormal(4, 1))) + 1

        # book state before this message
        cur_mid = _mid_from_l2(prev_l2, prev_mid)
        books[i, 0] = (cur_mid - prev_mid) / TICK
        books[i, 1] = ts
        books[i, 2] = tns
        books[i, 3:] = prev_l2
        p_ref = (cur_mid // TICK) * TICK

        own = ob.bids if side == 1 else ob.asks
        live = np.nonzero(own[:, 0] >= 0)[0]
        if et in (2, 3, 4) and len(live) == 0:
            et = 1
        ref = (NA_VAL, NA_VAL, NA_VAL, NA_VAL)
        if et == 1:
            off = int(np.clip(np.round(rng.laplace(0.0, 5.0)), -500, 500))
            price = (mid + off) * TICK
            oid = next_oid
            next_oid += 1
            qty = size
        else:
            if et == 4:
                top = ob._top_bid(own) if side == 1 else ob._top_ask(own)
                row = own[top]
                qty = int(min(size, row[1]))
            else:
                row = own[live[rng.integers(len(live))]]
                qty = int(row[1]) if et == 3 else (int(rng.integers(1, row[1])) if row[1] > 1 else 1)
            price, oid = int(row[0]), int(row[2])
            if oid in submitted:
                ref = submitted[oid]
        em = np.array([et, side, qty, price, oid, 0, ts, tns], dtype=np.int64)
        ob.process(em)
        emsgs[i] = em

        rel = int(np.clip((price - p_ref), -99900, 99900) // TICK)
        if et == 1:
            submitted[oid] = (rel, min(qty, 9999), ts, tns)
        msgs[i] = [oid, et, (side + 1) // 2, price, rel, min(qty, 9999),
                   dt // 10**9, dt % 10**9, ts, tns, *ref]
        prev_l2 = ob.l2(levels)
        prev_mid = cur_mid
    return SyntheticDay(msgs, books, emsgs, l2_0)


def make_sequences(n_seqs: int, n_msgs: int, seed: int = 0, levels: int = 10):
    """``n_seqs`` independent days of ``n_msgs`` messages each."""
    days = [generate_day(n_msgs, seed=seed * 100003 + k, levels=levels) for k in range(n_seqs)]
    return days
