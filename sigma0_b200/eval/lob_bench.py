"""LOB-Bench scoring: distributional distances between generated and real order flow.

The reference scores generated message streams against real ones with the LOB-Bench suite
(``src/lobpipeline/scorer/lob_bench/run_bench.py:20-215`` its default metric table,
``eval.py`` the statistics, ``metrics.py`` the bootstrapped distances, ``impact.py`` the
price-impact response functions).  This module computes the same families from this
package's arrays -- messages ``(n, >=7)`` ``[time_s, time_ns, type, order_id, size, price,
direction]`` and the L2 book after each message ``(n, 4L)`` ``[ask_p, ask_v, bid_p,
bid_v, ...]`` -- in numpy, with statistics written from their definitions.

Unconditional metrics (``METRICS``, 22): spread; L1 order-book imbalance; log inter-arrival
time; log time to cancel and to first fill (per order id); touch and 10-level volume per
side; depth (distance to the mid) of new limit orders and of cancellations per side; ticks
from the best price of new limit orders and of cancellations per side; executed volume
per minute; order-flow imbalance (rolling mean over 100 events) and its value before an
up / unchanged / down mid move.

Conditional metrics (``COND_METRICS``): a statistic within quantile bins of a conditioning
one (bins from the real data), the distance averaged over bins weighted by the real
data's bin shares: touch ask volume | spread, spread | time of day, spread | realized
volatility, touch ask / bid volume | order-flow imbalance.

Distances: L1 between normalised histograms (the discrete metrics on integer bins),
Wasserstein-1 and Kolmogorov-Smirnov, each with a bootstrap 95% interval.

Impact (``impact_responses``): the response function R(l) = E[s_t (m_{t+l} - m_t)] / tick of
each event class (market orders, limit orders and cancellations, each split by whether it
moved the touch) with sign s_t = +1 for buy-side pressure (buy market order, bid limit
order, ask cancellation), for lags l in events; ``impact_score`` compares the curves of two
streams.  The Cont-Stoikov-Talreja baseline generator is ``eval/cst.py``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from .lob_metrics import hist_l1, ks_stat, wasserstein1

LIMIT, CANCEL, DELETE, EXEC = 1, 2, 3, 4


def _t(m):
    return m[:, 0].astype(np.float64) + m[:, 1].astype(np.float64) * 1e-9


def _valid_touch(b):
    return (b[:, 0] > 0) & (b[:, 0] < 2e9) & (b[:, 2] > 0) & (b[:, 2] > -2e9)


def _mid(b):
    ok = _valid_touch(b)
    mid = np.where(ok, (b[:, 0].astype(np.float64) + b[:, 2]) / 2.0, np.nan)
    idx = np.where(ok, np.arange(len(mid)), 0)
    np.maximum.accumulate(idx, out=idx)
    return mid[idx]


def spread(m, b, tick=100):
    ok = _valid_touch(b)
    return (b[ok, 0] - b[ok, 2]) / tick


def imbalance(m, b, tick=100):
    return (b[:, 3] - b[:, 1]) / np.maximum(b[:, 1] + b[:, 3], 1)


def log_inter_arrival(m, b, tick=100):
    d = np.diff(_t(m))
    return np.log(d[d > 0])


def _first_after(m, types_start, types_end):
    """Per order id: time from its first message of ``types_start`` to its first later
    message of ``types_end``."""
    t = _t(m)
    oid, typ = m[:, 3], m[:, 2]
    start: Dict[int, float] = {}
    out = []
    for i in range(len(m)):
        o = int(oid[i])
        if typ[i] in types_start and o not in start:
            start[o] = t[i]
        elif typ[i] in types_end and o in start:
            out.append(t[i] - start.pop(o))
    a = np.asarray(out, np.float64)
    return np.log(a[a > 0])


def log_time_to_cancel(m, b, tick=100):
    return _first_after(m, (LIMIT,), (CANCEL, DELETE))


def log_time_to_first_fill(m, b, tick=100):
    return _first_after(m, (LIMIT,), (EXEC,))


def _depth(m, b, types):
    sel = np.isin(m[:, 2], types)
    d = m[sel, 5] - _mid(b)[sel]
    return d[d > 0], -d[d < 0]


def _ticks(m, b, types, tick):
    # cancellations are measured against the book before the message
    prev = np.vstack([b[:1], b[:-1]]) if np.isin(types, (CANCEL, DELETE)).any() else b
    sel = np.isin(m[:, 2], types) & _valid_touch(prev)
    p, ba, bb = m[sel, 5], prev[sel, 0], prev[sel, 2]
    mid = (ba + bb) / 2.0
    ask = p >= mid
    return (np.clip(np.round((p[ask] - ba[ask]) / tick), 0, None),
            np.clip(np.round((bb[~ask] - p[~ask]) / tick), 0, None))


def vol_per_min(m, b, tick=100):
    ex = m[:, 2] == EXEC
    if not ex.any():
        return np.zeros(0)
    t = _t(m)[ex]
    sec = np.floor(t)
    uniq, inv = np.unique(sec, return_inverse=True)
    vol = np.bincount(inv, weights=m[ex, 4].astype(np.float64))
    if len(uniq) > 2:                       # edge seconds are partial: dropped
        vol = vol[1:-1]
    return vol * 60.0


def ofi(m, b, tick=100, window=100):
    ap, av, bp, bv = (b[:, i].astype(np.float64) for i in range(4))
    da, db = np.diff(ap), np.diff(bp)
    e = ((db >= 0) * bv[1:] - (db <= 0) * bv[:-1] - (da <= 0) * av[1:] + (da >= 0) * av[:-1])
    if len(e) < window:
        return np.zeros(0)
    c = np.cumsum(np.concatenate([[0.0], e]))
    return (c[window:] - c[:-window]) / window


def _ofi_before(m, b, tick, sign, window=100):
    o = ofi(m, b, tick, window)
    if len(o) < 2:
        return np.zeros(0)
    dm = np.sign(np.diff(_mid(b)))[window:]
    n = min(len(o) - 1, len(dm))
    prev, d = o[:n], dm[:n]
    return prev[d == sign]


METRICS: Dict[str, Tuple[Callable, bool]] = {
    "spread": (spread, True),
    "orderbook_imbalance": (imbalance, False),
    "log_inter_arrival_time": (log_inter_arrival, False),
    "log_time_to_cancel": (log_time_to_cancel, False),
    "log_time_to_first_fill": (log_time_to_first_fill, False),
    "ask_volume_touch": (lambda m, b, tick=100: b[:, 1].astype(np.float64), False),
    "bid_volume_touch": (lambda m, b, tick=100: b[:, 3].astype(np.float64), False),
    "ask_volume": (lambda m, b, tick=100: b[:, 1::4][:, :10].sum(1).astype(np.float64), False),
    "bid_volume": (lambda m, b, tick=100: b[:, 3::4][:, :10].sum(1).astype(np.float64), False),
    "limit_ask_order_depth": (lambda m, b, tick=100: _depth(m, b, (LIMIT,))[0], False),
    "limit_bid_order_depth": (lambda m, b, tick=100: _depth(m, b, (LIMIT,))[1], False),
    "ask_cancellation_depth": (lambda m, b, tick=100: _depth(m, b, (CANCEL, DELETE))[0], False),
    "bid_cancellation_depth": (lambda m, b, tick=100: _depth(m, b, (CANCEL, DELETE))[1], False),
    "limit_ask_order_ticks": (lambda m, b, tick=100: _ticks(m, b, (LIMIT,), tick)[0], True),
    "limit_bid_order_ticks": (lambda m, b, tick=100: _ticks(m, b, (LIMIT,), tick)[1], True),
    "ask_cancellation_ticks": (lambda m, b, tick=100: _ticks(m, b, (CANCEL, DELETE), tick)[0], True),
    "bid_cancellation_ticks": (lambda m, b, tick=100: _ticks(m, b, (CANCEL, DELETE), tick)[1], True),
    "vol_per_min": (vol_per_min, False),
    "ofi": (ofi, False),
    "ofi_up": (lambda m, b, tick=100: _ofi_before(m, b, tick, 1), False),
    "ofi_stay": (lambda m, b, tick=100: _ofi_before(m, b, tick, 0), False),
    "ofi_down": (lambda m, b, tick=100: _ofi_before(m, b, tick, -1), False),
}


def _time_of_day(m, b, tick=100):
    return np.floor((m[:, 0].astype(np.float64) % 86400) / 1800.0)      # half-hour buckets


def _volatility(m, b, tick=100):
    """Realised volatility of log mid returns over the stream (one value per message)."""
    mid = _mid(b)
    r = np.diff(np.log(mid[np.isfinite(mid)]))
    v = float(np.sqrt(np.sum(r * r))) if len(r) else 0.0
    return np.full(len(m), v)


def _aligned(eval_fn, cond_fn):
    """(eval, cond) sequences of equal length (aligned at the end: rolling statistics start later)."""
    def f(m, b, tick=100):
        e, c = np.asarray(eval_fn(m, b, tick), float), np.asarray(cond_fn(m, b, tick), float)
        n = min(len(e), len(c))
        return e[len(e) - n:], c[len(c) - n:]
    return f


COND_METRICS: Dict[str, Callable] = {
    "ask_volume_touch|spread": _aligned(METRICS["ask_volume_touch"][0], lambda m, b, tick=100:
                                        (b[:, 0] - b[:, 2]) / tick),
    "spread|time_of_day": _aligned(lambda m, b, tick=100: (b[:, 0] - b[:, 2]) / tick, _time_of_day),
    "spread|volatility": _aligned(lambda m, b, tick=100: (b[:, 0] - b[:, 2]) / tick, _volatility),
    "ask_volume_touch|ofi": _aligned(METRICS["ask_volume_touch"][0], ofi),
    "bid_volume_touch|ofi": _aligned(METRICS["bid_volume_touch"][0], ofi),
}


def compute(msgs_list: Sequence[np.ndarray], books_list: Sequence[np.ndarray], tick: int = 100,
            metrics: Optional[Sequence[str]] = None) -> Dict[str, np.ndarray]:
    """Every unconditional metric over a set of streams (values concatenated)."""
    names = list(metrics) if metrics is not None else list(METRICS)
    out = {k: [] for k in names}
    for m, b in zip(msgs_list, books_list):
        m, b = np.asarray(m), np.asarray(b)
        for k in names:
            v = np.asarray(METRICS[k][0](m, b, tick), np.float64)
            out[k].append(v[np.isfinite(v)])
    return {k: (np.concatenate(v) if v else np.zeros(0)) for k, v in out.items()}


def compute_conditional(msgs_list, books_list, tick: int = 100) -> Dict[str, Tuple[np.ndarray, np.ndarray]]:
    out = {}
    for k, fn in COND_METRICS.items():
        es, cs = [], []
        for m, b in zip(msgs_list, books_list):
            e, c = fn(np.asarray(m), np.asarray(b), tick)
            ok = np.isfinite(e) & np.isfinite(c)
            es.append(e[ok])
            cs.append(c[ok])
        out[k] = (np.concatenate(es) if es else np.zeros(0), np.concatenate(cs) if cs else np.zeros(0))
    return out


def _discrete_l1(a, b):
    if not len(a) or not len(b):
        return float("nan")
    lo, hi = int(min(a.min(), b.min())), int(max(a.max(), b.max()))
    ha = np.bincount((a - lo).astype(int), minlength=hi - lo + 1) / len(a)
    hb = np.bincount((b - lo).astype(int), minlength=hi - lo + 1) / len(b)
    return float(np.abs(ha - hb).sum())


@dataclass
class BenchScore:
    metric: str
    distance: str
    value: float
    ci_low: float
    ci_high: float


def _boot(fn, a, b, n_boot, rng):
    v = fn(a, b)
    if len(a) < 2 or len(b) < 2 or n_boot <= 0:
        return v, v, v
    bs = [fn(rng.choice(a, len(a)), rng.choice(b, len(b))) for _ in range(n_boot)]
    lo, hi = np.nanpercentile(bs, [2.5, 97.5])
    return v, float(lo), float(hi)


def score_unconditional(gen: Dict[str, np.ndarray], real: Dict[str, np.ndarray], n_boot: int = 50, seed: int = 0,
                        max_samples: int = 20_000) -> List[BenchScore]:
    rng = np.random.default_rng(seed)
    out = []
    for k in gen:
        if k not in real:
            continue
        a, b = gen[k], real[k]
        if len(a) > max_samples:
            a = rng.choice(a, max_samples, replace=False)
        if len(b) > max_samples:
            b = rng.choice(b, max_samples, replace=False)
        discrete = METRICS[k][1] if k in METRICS else False
        l1 = _discrete_l1 if discrete else hist_l1
        for name, fn in (("l1", l1), ("wasserstein", wasserstein1), ("ks", ks_stat)):
            v, lo, hi = _boot(fn, a, b, n_boot if name == "l1" else min(n_boot, 20), rng)
            out.append(BenchScore(k, name, v, lo, hi))
    return out


def score_conditional(gen, real, n_bins: int = 5) -> List[BenchScore]:
    """Per conditional metric: the L1 / Wasserstein distance of the evaluated statistic
    within each quantile bin of the condition (bins from the real data), weighted by the
    real bin shares."""
    out = []
    for k in gen:
        if k not in real:
            continue
        (ge, gc), (re, rc) = gen[k], real[k]
        if not len(re) or not len(ge):
            continue
        edges = np.unique(np.quantile(rc, np.linspace(0, 1, n_bins + 1)))
        if len(edges) < 2:
            edges = np.array([rc.min() - 0.5, rc.max() + 0.5])
        gi = np.clip(np.searchsorted(edges, gc, side="right") - 1, 0, len(edges) - 2)
        ri = np.clip(np.searchsorted(edges, rc, side="right") - 1, 0, len(edges) - 2)
        tot_l1 = tot_w = wsum = 0.0
        for j in range(len(edges) - 1):
            a, b = ge[gi == j], re[ri == j]
            if not len(b):
                continue
            w = len(b) / len(re)
            if len(a):
                tot_l1 += w * hist_l1(a, b)
                tot_w += w * wasserstein1(a, b)
            else:
                tot_l1 += w * 2.0                 # nothing generated in this bin: maximal L1
                tot_w += w * float(np.std(b))
            wsum += w
        out.append(BenchScore(k, "l1", tot_l1 / max(wsum, 1e-12), float("nan"), float("nan")))
        out.append(BenchScore(k, "wasserstein", tot_w / max(wsum, 1e-12), float("nan"), float("nan")))
    return out


# ---- price impact -------------------------------------------------------------------------------
def _event_classes(m, b):
    """Per message: (class name or None, sign).  Classes: MO0/MO1 (market orders that left /
    moved the touch), LO0/LO1 (limit orders outside / inside the spread), CA0/CA1
    (cancellations that left / emptied the touch level)."""
    prev = np.vstack([b[:1], b[:-1]])
    typ, price, dirn = m[:, 2], m[:, 5], m[:, 6]
    moved = (b[:, 0] != prev[:, 0]) | (b[:, 2] != prev[:, 2])
    cls = np.full(len(m), None, dtype=object)
    sign = np.zeros(len(m))
    ex = typ == EXEC
    # an execution of a resting order on side d is a market order of the opposite sign
    cls[ex] = np.where(moved[ex], "MO1", "MO0")
    sign[ex] = -dirn[ex]
    lo = typ == LIMIT
    inside = (price < prev[:, 0]) & (price > prev[:, 2])
    cls[lo] = np.where(inside[lo], "LO1", "LO0")
    sign[lo] = dirn[lo]
    ca = np.isin(typ, (CANCEL, DELETE))
    cls[ca] = np.where(moved[ca], "CA1", "CA0")
    sign[ca] = -dirn[ca]
    return cls, sign


def impact_responses(msgs_list, books_list, lags: Sequence[int] = (1, 2, 5, 10, 20, 50, 100),
                     tick: int = 100) -> Dict[str, np.ndarray]:
    """R(l) per event class: the mean signed mid change (ticks) l events after the event."""
    acc: Dict[str, List[np.ndarray]] = {}
    for m, b in zip(msgs_list, books_list):
        m, b = np.asarray(m), np.asarray(b)
        mid = _mid(b)
        cls, sign = _event_classes(m, b)
        for c in ("MO0", "MO1", "LO0", "LO1", "CA0", "CA1"):
            idx = np.nonzero(cls == c)[0]
            rows = []
            for lag in lags:
                j = idx[idx + lag < len(mid)]
                if len(j):
                    d = (mid[j + lag] - mid[j]) / tick * sign[j]
                    rows.append(float(np.nanmean(d)))
                else:
                    rows.append(np.nan)
            acc.setdefault(c, []).append(np.asarray(rows))
    return {c: np.nanmean(np.stack(v), 0) for c, v in acc.items()}


def impact_score(gen: Dict[str, np.ndarray], real: Dict[str, np.ndarray]) -> Dict[str, float]:
    """Mean absolute difference of the response curves (ticks), per class and overall."""
    out = {}
    for c in real:
        if c in gen:
            d = np.abs(gen[c] - real[c])
            out[c] = float(np.nanmean(d)) if np.isfinite(d).any() else float("nan")
    vals = [v for v in out.values() if np.isfinite(v)]
    out["mean"] = float(np.mean(vals)) if vals else float("nan")
    return out


def run_bench(gen_msgs, gen_books, real_msgs, real_books, tick: int = 100, n_boot: int = 50,
              seed: int = 0) -> Dict:
    """Every score of this module for one generated / real pair of stream sets."""
    g, r = compute(gen_msgs, gen_books, tick), compute(real_msgs, real_books, tick)
    gc, rc = compute_conditional(gen_msgs, gen_books, tick), compute_conditional(real_msgs, real_books, tick)
    return {
        "unconditional": score_unconditional(g, r, n_boot=n_boot, seed=seed),
        "conditional": score_conditional(gc, rc),
        "impact": impact_score(impact_responses(gen_msgs, gen_books, tick=tick),
                               impact_responses(real_msgs, real_books, tick=tick)),
    }
