"""Generated-vs-real order-flow statistics (LOB-Bench style) and the return bench.

* ``validity_report`` -- the semantic checks applied to every generated window:
  timestamps non-decreasing, nanoseconds in range, all values finite, events in
  {1..4}, sides in {-1, 1}, sizes positive (``docs/inference.md`` "Validity").
* ``marginals`` -- per-window scalar series that the LOB-Bench scorer compares
  (spread, mid log-returns, inter-arrival times, order sizes, level-1 depth,
  order-book imbalance, event-type shares, limit-order distance to the mid);
  ``score`` computes Wasserstein-1, Kolmogorov-Smirnov and histogram-L1 distances
  between generated and real samples, with bootstrap confidence intervals
  (the reference vendors LOB-Bench; ``lobpipeline/scorer``).
* ``event_returns`` -- the return bench (``lobpipeline/return_bench/run_event_bench.py``):
  mid-price return at fixed wall-clock horizons after each anchor event, with a
  shuffled-anchor null for comparison.

Inputs are the arrays the generator emits (messages ``[time_s, time_ns, type,
oid, size, price, direction]`` and L2 rows) or the CSVs the inference CLI writes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np


# ---------------------------------------------------------------------------
# validity
# ---------------------------------------------------------------------------

def validity_report(msgs: np.ndarray) -> Dict[str, int]:
    """msgs (n, >=7) [time_s, time_ns, type, oid, size, price, direction] -> violation counts."""
    m = np.asarray(msgs, dtype=np.float64)
    t = m[:, 0] * 1e9 + m[:, 1]
    return {
        "n": int(len(m)),
        "non_monotone_time": int(np.sum(np.diff(t) < 0)),
        "ns_out_of_range": int(np.sum((m[:, 1] < 0) | (m[:, 1] >= 1e9))),
        "non_finite": int(np.sum(~np.isfinite(m))),
        "bad_event_type": int(np.sum(~np.isin(m[:, 2], [1, 2, 3, 4]))),
        "bad_side": int(np.sum(~np.isin(m[:, 6], [-1, 1]))),
        "non_positive_size": int(np.sum(m[:, 4] <= 0)),
    }


# ---------------------------------------------------------------------------
# marginals
# ---------------------------------------------------------------------------

def _mid(l2: np.ndarray) -> np.ndarray:
    ap, bp = l2[:, 0].astype(np.float64), l2[:, 2].astype(np.float64)
    ok = (ap > 0) & (bp > 0) & (ap < 2e9) & (bp > -2e9)
    mid = np.where(ok, (ap + bp) / 2, np.nan)
    # carry the last valid mid over one-sided books
    idx = np.where(ok, np.arange(len(mid)), 0)
    np.maximum.accumulate(idx, out=idx)
    return mid[idx]


def marginals(msgs: np.ndarray, l2: np.ndarray, tick: int = 100) -> Dict[str, np.ndarray]:
    m = np.asarray(msgs, dtype=np.float64)
    b = np.asarray(l2, dtype=np.float64)
    mid = _mid(b)
    t = m[:, 0] + m[:, 1] * 1e-9
    spread = (b[:, 0] - b[:, 2]) / tick
    spread = spread[(b[:, 0] < 2e9) & (b[:, 2] > -2e9)]
    depth1 = b[:, 1] + b[:, 3]
    imb = (b[:, 3] - b[:, 1]) / np.maximum(b[:, 1] + b[:, 3], 1)
    lim = m[:, 2] == 1
    dist = np.abs(m[lim, 5] - mid[lim]) / tick if lim.any() else np.zeros(0)
    out = {
        "spread_ticks": spread,
        "mid_logret": np.diff(np.log(mid[np.isfinite(mid)])) if np.isfinite(mid).sum() > 1 else np.zeros(0),
        "interarrival_s": np.diff(t),
        "order_size": m[:, 4],
        "depth_l1": depth1,
        "imbalance_l1": imb,
        "limit_distance_ticks": dist,
    }
    for e in (1, 2, 3, 4):
        out[f"share_type_{e}"] = np.array([float(np.mean(m[:, 2] == e))])
    return out


def wasserstein1(a: np.ndarray, b: np.ndarray) -> float:
    from scipy.stats import wasserstein_distance
    return float(wasserstein_distance(a, b)) if len(a) and len(b) else float("nan")


def ks_stat(a: np.ndarray, b: np.ndarray) -> float:
    from scipy.stats import ks_2samp
    return float(ks_2samp(a, b).statistic) if len(a) and len(b) else float("nan")


def hist_l1(a: np.ndarray, b: np.ndarray, bins: int = 50) -> float:
    if not len(a) or not len(b):
        return float("nan")
    lo, hi = np.nanmin(np.concatenate([a, b])), np.nanmax(np.concatenate([a, b]))
    if hi <= lo:
        return 0.0
    ha, _ = np.histogram(a, bins=bins, range=(lo, hi))
    hb, _ = np.histogram(b, bins=bins, range=(lo, hi))
    return float(np.abs(ha / ha.sum() - hb / hb.sum()).sum())


@dataclass
class Score:
    metric: str
    value: float
    ci_low: float
    ci_high: float


def score(gen: Dict[str, np.ndarray], real: Dict[str, np.ndarray], n_boot: int = 100, seed: int = 0,
          distances=("wasserstein", "ks", "l1")) -> List[Score]:
    """Distances between generated and real marginals, with bootstrap 95% intervals."""
    fns = {"wasserstein": wasserstein1, "ks": ks_stat, "l1": hist_l1}
    rng = np.random.default_rng(seed)
    out = []
    for key in sorted(set(gen) & set(real)):
        a, b = np.asarray(gen[key], float), np.asarray(real[key], float)
        a, b = a[np.isfinite(a)], b[np.isfinite(b)]
        for d in distances:
            v = fns[d](a, b)
            boots = []
            if len(a) > 1 and len(b) > 1:
                for _ in range(n_boot):
                    boots.append(fns[d](rng.choice(a, len(a)), rng.choice(b, len(b))))
            lo, hi = (np.percentile(boots, [2.5, 97.5]) if boots else (v, v))
            out.append(Score(f"{key}/{d}", v, float(lo), float(hi)))
    return out


def concat_marginals(parts: Iterable[Dict[str, np.ndarray]]) -> Dict[str, np.ndarray]:
    acc: Dict[str, List[np.ndarray]] = {}
    for p in parts:
        for k, v in p.items():
            acc.setdefault(k, []).append(np.asarray(v, float))
    return {k: np.concatenate(v) for k, v in acc.items()}


# ---------------------------------------------------------------------------
# return bench
# ---------------------------------------------------------------------------

def event_returns(msgs: np.ndarray, l2: np.ndarray, anchor_types: Sequence[int] = (4,),
                  horizons_ms: Sequence[float] = (10, 100, 1000), side_sign: bool = True,
                  shuffle_seed: Optional[int] = 0) -> Dict[str, Dict[float, float]]:
    """Mean mid log-return (bps) at wall-clock horizons after anchor events, signed by the
    anchor's side when ``side_sign``; ``null`` uses shuffled anchor times."""
    m = np.asarray(msgs, dtype=np.float64)
    t = m[:, 0] + m[:, 1] * 1e-9
    mid = _mid(np.asarray(l2, dtype=np.float64))

    def at(times):
        idx = np.searchsorted(t, times, side="right") - 1
        idx = np.clip(idx, 0, len(t) - 1)
        return mid[idx]
    anc = np.isin(m[:, 2], anchor_types)
    sign = np.where(m[:, 6] > 0, 1.0, -1.0) if side_sign else np.ones(len(m))

    def mean_ret(idx):
        res = {}
        for h in horizons_ms:
            r = (np.log(at(t[idx] + h / 1000.0)) - np.log(mid[idx])) * 1e4 * sign[idx]
            r = r[np.isfinite(r)]
            res[h] = float(r.mean()) if len(r) else float("nan")
        return res
    idx = np.nonzero(anc)[0]
    out = {"anchors": {0: float(len(idx))}, "event": mean_ret(idx)}
    if shuffle_seed is not None and len(idx):
        rng = np.random.default_rng(shuffle_seed)
        out["null"] = mean_ret(rng.choice(len(m), len(idx), replace=False))
    return out
