"""Replay fidelity of the market-making simulator: how faithfully a message stream replays
through the matching engine from the conditioning book.

The reference keeps two arms apart (``src/post_training/heuristic_learning/fidelity.py:1-120``):
the real arm replays the REAL continuation from the real conditioning book and compares the
book path with the recorded one; the gen arm replays the GENERATED continuation and compares
with the book the generator recorded.  Both run the same code, so a divergence in the real arm
is the simulator's own (initialisation, id resolution) and one only in the gen arm is the
generator's.  Every replay carries a report of what could not be applied exactly
(``ReplayReport``, ``:131-190``) next to the agreement numbers (``compare_paths``, ``:324``):
a simulator that silently absorbs messages it could not apply produces a plausible PnL from a
market that never existed.

Messages here are engine rows ``(type, side, size, price, order_id, trader_id, time_s,
time_ns)``; books are L2 rows ``[ask_p, ask_v, bid_p, bid_v, ...]``, row i the book AFTER
message i (the preprocessed data layout stores the book before each message: pass its rows
shifted by one).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Dict, Optional, Sequence, Tuple

import numpy as np

from ..engine.book import NEGATIVE_RETURN_ID, EngineConfig, OrderBook, init_msgs_from_l2


@dataclass
class ReplayReport:
    n_messages: int = 0
    span_s: float = 0.0
    monotonic: bool = True
    n_negative_deltas: int = 0
    event_types: Dict[int, int] = field(default_factory=dict)
    n_unhandled_types: int = 0
    n_cancel_delete: int = 0
    n_unresolvable_ids: int = 0
    n_unresolved_positive: int = 0      # an id never seen and not an init order: the price fallback
    n_lookup_miss_sentinel: int = 0     # the generator's own lookup failed
    n_init_ref_in_depth: int = 0        # names an init order this replay creates
    n_init_ref_out_of_depth: int = 0    # names an init order deeper than this replay's book
    first_bad_id_step: int = -1

    @property
    def clean(self) -> bool:
        return self.monotonic and self.n_unhandled_types == 0

    def as_dict(self) -> Dict:
        d = asdict(self)
        d["clean"] = self.clean
        return d


def describe_stream(msgs: np.ndarray, prior_ids: Optional[Sequence[int]] = None, n_levels: int = 10,
                    cfg: EngineConfig = EngineConfig()) -> ReplayReport:
    """Diagnose a stream without running it: timing, event types, and every cancel / delete
    whose order id the replay cannot resolve, split by why."""
    m = np.asarray(msgs, np.int64)
    r = ReplayReport(n_messages=len(m))
    if not len(m):
        return r
    t = m[:, 6].astype(np.float64) + m[:, 7].astype(np.float64) * 1e-9
    dt = np.diff(t)
    r.span_s = float(t[-1] - t[0])
    r.n_negative_deltas = int((dt < 0).sum())
    r.monotonic = r.n_negative_deltas == 0
    types, counts = np.unique(m[:, 0], return_counts=True)
    r.event_types = {int(a): int(b) for a, b in zip(types, counts)}
    r.n_unhandled_types = int((~np.isin(m[:, 0], (1, 2, 3, 4))).sum())
    known = set(int(x) for x in (prior_ids or ()))
    lo_in, hi_in = cfg.init_id - (2 * n_levels - 1), cfg.init_id
    lo_all = cfg.init_id - (2 * cfg.book_depth - 1)
    for i, row in enumerate(m):
        typ, oid = int(row[0]), int(row[4])
        if typ == 1:
            known.add(oid)
            continue
        if typ not in (2, 3):
            continue
        r.n_cancel_delete += 1
        if oid in known:
            continue
        if oid == NEGATIVE_RETURN_ID:
            r.n_lookup_miss_sentinel += 1
            bad = True
        elif lo_in <= oid <= hi_in:
            r.n_init_ref_in_depth += 1
            bad = False
        elif lo_all <= oid < lo_in:
            r.n_init_ref_out_of_depth += 1
            bad = True
        else:
            r.n_unresolved_positive += 1
            bad = False
        r.n_unresolvable_ids += 1
        if bad and r.first_bad_id_step < 0:
            r.first_bad_id_step = i
    return r


def replay_stream(msgs: np.ndarray, init_l2: np.ndarray, n_levels: int = 10,
                  cfg: EngineConfig = EngineConfig(), time=(34200, 0)) -> Tuple[np.ndarray, ReplayReport]:
    """Rebuild the book from ``init_l2`` and replay ``msgs``; the L2 path after each message
    (``n_levels`` levels) and the stream's report."""
    ob = OrderBook(cfg)
    init = init_msgs_from_l2(np.asarray(init_l2, np.int64), cfg, time)
    for row in init:
        ob.process(row)
    prior = [int(x) for x in init[:, 4]]
    rep = describe_stream(msgs, prior, n_levels=np.asarray(init_l2).shape[0] // 4, cfg=cfg)
    path = np.zeros((len(msgs), 4 * n_levels), np.int64)
    for i, row in enumerate(np.asarray(msgs, np.int64)):
        ob.process(row)
        path[i] = ob.l2(n_levels)
    return path, rep


def mid_from_book(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.float64)[:, 0] + np.asarray(b, np.float64)[:, 2]) / 2.0


def compare_paths(ours: np.ndarray, reference: np.ndarray, tick: int = 100) -> Dict[str, float]:
    """Per-step agreement of two book paths: whole rows equal, mids equal, the mean absolute
    mid difference (ticks) and the first step where the rows differ (-1: never)."""
    n = min(len(ours), len(reference))
    if n == 0:
        return {"exact_full_frac": 0.0, "exact_mid_frac": 0.0, "mean_abs_mid_ticks": float("nan"),
                "first_divergence": -1}
    w = min(ours.shape[1], reference.shape[1])
    eq = (np.asarray(ours)[:n, :w] == np.asarray(reference)[:n, :w]).all(1)
    d = np.abs(mid_from_book(ours[:n]) - mid_from_book(reference[:n])) / tick
    first = int(np.argmin(eq)) if not eq.all() else -1
    return {"exact_full_frac": float(eq.mean()), "exact_mid_frac": float((d == 0).mean()),
            "mean_abs_mid_ticks": float(d.mean()), "first_divergence": first}


def window_report(init_l2: np.ndarray, real_msgs: np.ndarray, real_books: np.ndarray,
                  gen_msgs: Optional[np.ndarray] = None, gen_books: Optional[np.ndarray] = None,
                  n_levels: int = 10, tick: int = 100) -> Dict[str, Dict]:
    """Both arms for one conditioning window."""
    out = {}
    arms = [("real", real_msgs, real_books)]
    if gen_msgs is not None and gen_books is not None:
        arms.append(("gen", gen_msgs, gen_books))
    for name, m, b in arms:
        path, rep = replay_stream(m, init_l2, n_levels)
        out[name] = {**compare_paths(path, np.asarray(b, np.int64)[:, :4 * n_levels], tick), **rep.as_dict()}
    return out
