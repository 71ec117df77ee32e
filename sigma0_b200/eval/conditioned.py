"""Conditioned fidelity breakdowns of generated order flow: tails, regimes, position in window.

The analyse-only breakdowns of the reference's ``tools/diagnostics/lob_evals.py``
(``eval_tail_conditioned`` :359, ``eval_regime_stratified`` :406,
``eval_position_in_window`` :759, ``fit_cg_surface`` :820), written here over plain
arrays.  The result keys are the reference's, so tables from the two compare:

* ``dense_features(msgs, book)`` -- per-message feature series of one window (spread,
  total and touch volumes per side, touch imbalance, signed order flow, log inter-arrival
  time, limit-order depth per side in ticks from the same-side touch);
* ``tail_conditioned`` -- per feature, W1 over the whole distribution and over the mass
  above the real q-quantile, raw and normalised by the mean absolute real value of that
  region, their ratios, and gen / real q-quantile ratios;
* ``regime_stratified`` -- windows split into tertiles of the real window's realised
  volatility and median spread; per tertile the mean W1 of the dense features and the
  Spearman correlation of generated vs real window log-returns (with a window-bootstrap
  interval), plus the spread of the IC across tertiles;
* ``position_in_window`` -- fixed-width bins of the position tau inside the generated
  window: W1 of generated vs real rows at the same tau (and vs all real rows), and the fit
  WS_tau = alpha + beta * tau^p;
* ``fit_cg_surface`` -- alpha across conditioning lengths c and c*, the smallest c whose
  normalised residual (alpha(c) - alpha(c_max)) / (alpha(0) - alpha(c_max)) is below 0.1.

W1 is the L1 distance between the two empirical quantile functions on a common grid
(W1 = integral over u of |F^-1(u) - G^-1(u)|).
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import numpy as np

EMPTY = 2_000_000_000
DENSE_FEATURES = ("spread", "ask_volume", "bid_volume", "ask_volume_touch", "bid_volume_touch",
                  "orderbook_imbalance", "ofi", "log_inter_arrival_time")


def w1(a, b, n_grid: int = 4000) -> float:
    a = np.sort(np.asarray(a, dtype=np.float64).ravel())
    b = np.sort(np.asarray(b, dtype=np.float64).ravel())
    a, b = a[np.isfinite(a)], b[np.isfinite(b)]
    if a.size == 0 or b.size == 0:
        return float("nan")
    m = min(a.size, b.size, n_grid)
    u = (np.arange(m) + 0.5) / m
    qa = np.interp(u * (a.size - 1), np.arange(a.size), a)
    qb = np.interp(u * (b.size - 1), np.arange(b.size), b)
    return float(np.mean(np.abs(qa - qb)))


# ---------------------------------------------------------------------------
# features
# ---------------------------------------------------------------------------

def dense_features(msgs: np.ndarray, book: np.ndarray, tick: float = 100.0) -> Dict[str, np.ndarray]:
    """msgs (n, >=7) [time_s, time_ns, type, oid, size, price, direction], book (n, 4 * levels)
    [ask_p, ask_v, bid_p, bid_v, ...] after each message -> {feature: (n,)} (NaN where a
    feature is undefined, e.g. a one-sided book or a non-limit event)."""
    m = np.asarray(msgs, dtype=np.float64)
    b = np.asarray(book, dtype=np.float64)
    n = min(len(m), len(b))
    m, b = m[:n], b[:n]
    ap, av, bp, bv = b[:, 0::4], b[:, 1::4], b[:, 2::4], b[:, 3::4]
    valid_a = (np.abs(ap) < EMPTY) & (ap > 0)
    valid_b = (np.abs(bp) < EMPTY) & (bp > 0)
    touch = valid_a[:, 0] & valid_b[:, 0]
    spread = np.where(touch, (ap[:, 0] - bp[:, 0]) / tick, np.nan)
    askv = np.where(valid_a, av, 0.0).sum(1)
    bidv = np.where(valid_b, bv, 0.0).sum(1)
    at = np.where(valid_a[:, 0], av[:, 0], 0.0)
    bt = np.where(valid_b[:, 0], bv[:, 0], 0.0)
    imb = np.where(at + bt > 0, (bt - at) / np.maximum(at + bt, 1e-12), np.nan)
    etype, size, side = m[:, 2], m[:, 4], m[:, 6]
    # signed flow: a limit order adds on its side, a cancel / deletion / execution removes
    sgn = np.where(side > 0, 1.0, -1.0)
    ofi = np.where(etype == 1, sgn * size, np.where(np.isin(etype, (2, 3, 4)), -sgn * size, 0.0))
    t = m[:, 0] + m[:, 1] * 1e-9
    dt = np.diff(t, prepend=t[0] if n else 0.0)
    lia = np.where(dt > 0, np.log(np.maximum(dt, 1e-12)), np.nan)
    price = m[:, 5]
    lim = etype == 1
    bid_touch, ask_touch = np.where(valid_b[:, 0], bp[:, 0], np.nan), np.where(valid_a[:, 0], ap[:, 0], np.nan)
    lbd = np.where(lim & (side > 0), (bid_touch - price) / tick, np.nan)
    lad = np.where(lim & (side < 0), (price - ask_touch) / tick, np.nan)
    return {"spread": spread, "ask_volume": askv, "bid_volume": bidv, "ask_volume_touch": at,
            "bid_volume_touch": bt, "orderbook_imbalance": imb, "ofi": ofi, "log_inter_arrival_time": lia,
            "limit_bid_order_depth": lbd, "limit_ask_order_depth": lad}


def stack_windows(per_window: Sequence[Dict[str, np.ndarray]], win_len: Optional[int] = None) -> Dict[str, np.ndarray]:
    """[{feature: (n_i,)}] -> {feature: (n_windows, win_len)} (windows cut / NaN-padded)."""
    if not per_window:
        return {}
    L = win_len or min(len(next(iter(w.values()))) for w in per_window)
    out = {}
    for f in per_window[0]:
        M = np.full((len(per_window), L), np.nan)
        for i, w in enumerate(per_window):
            v = w[f][:L]
            M[i, :len(v)] = v
        out[f] = M
    return out


def _pooled(x: np.ndarray) -> np.ndarray:
    v = np.asarray(x, dtype=np.float64).ravel()
    return v[np.isfinite(v)]


# ---------------------------------------------------------------------------
# tails
# ---------------------------------------------------------------------------

def tail_conditioned(real: Dict[str, np.ndarray], gen: Dict[str, np.ndarray],
                     quantiles: Sequence[float] = (0.90, 0.99)) -> Dict:
    res = {}
    for f in real:
        if f not in gen:
            continue
        r, g = _pooled(real[f]), _pooled(gen[f])
        if r.size == 0 or g.size == 0:
            continue
        ws = w1(r, g)
        rbar = float(np.mean(np.abs(r)))
        ws_norm = ws / rbar if rbar > 1e-12 else None
        row = {"ws_bulk": ws, "ws_bulk_norm": ws_norm}
        for q in quantiles:
            thr = np.quantile(r, q)
            rt, gt = r[r >= thr], g[g >= thr]
            wt = w1(rt, gt)
            tbar = float(np.mean(np.abs(rt))) if rt.size else float("nan")
            wt_norm = wt / tbar if (rt.size and tbar > 1e-12) else None
            qr, qg = float(np.quantile(r, q)), float(np.quantile(g, q))
            row[f"ws_tail_{q}"] = wt
            row[f"ratio_{q}"] = wt / ws if ws > 1e-12 else None
            row[f"ws_tail_{q}_norm"] = wt_norm
            row[f"ratio_{q}_norm"] = (wt_norm / ws_norm) if (ws_norm and wt_norm is not None and ws_norm > 1e-12) else None
            row[f"qratio_{q}"] = qg / qr if abs(qr) > 1e-12 else None
            row[f"n_real_tail_{q}"] = int(rt.size)
            row[f"n_gen_tail_{q}"] = int(gt.size)
        res[f] = row
    return {"eval": "tail_conditioned", "features": res}


# ---------------------------------------------------------------------------
# regimes
# ---------------------------------------------------------------------------

def _mid(book: np.ndarray) -> np.ndarray:
    b = np.asarray(book, dtype=np.float64)
    return (b[:, 0] + b[:, 2]) / 2.0


def _spearman(a: np.ndarray, b: np.ndarray) -> float:
    from scipy.stats import spearmanr
    ok = np.isfinite(a) & np.isfinite(b)
    if ok.sum() <= 2:
        return float("nan")
    return float(spearmanr(a[ok], b[ok]).statistic)


def _tertiles(x: np.ndarray) -> np.ndarray:
    lab = np.full(len(x), -1)
    good = np.isfinite(x)
    if good.sum() < 3:
        return lab
    q1, q2 = np.percentile(x[good], [33.3, 66.7])
    lab[good] = np.where(x[good] <= q1, 0, np.where(x[good] <= q2, 1, 2))
    return lab


def regime_stratified(books_real: Sequence[np.ndarray], books_gen: Sequence[np.ndarray],
                      dense_real: Dict[str, np.ndarray], dense_gen: Dict[str, np.ndarray],
                      ws_features: Sequence[str] = ("spread", "ask_volume", "bid_volume", "ask_volume_touch",
                                                    "bid_volume_touch", "orderbook_imbalance"),
                      n_boot: int = 200, seed: int = 0) -> Dict:
    n = min(len(books_real), len(books_gen))
    if n == 0:
        return {"eval": "regime_stratified", "status": "no windows"}
    spread, vol, rr, rg = (np.full(n, np.nan) for _ in range(4))
    for i in range(n):
        br, bg = np.asarray(books_real[i], dtype=np.float64), np.asarray(books_gen[i], dtype=np.float64)
        if br.shape[1] < 3 or bg.shape[1] < 3 or len(br) < 2 or len(bg) < 2:
            continue
        mr, mg = np.clip(_mid(br), 1e-9, None), np.clip(_mid(bg), 1e-9, None)
        spread[i] = float(np.median(br[:, 0] - br[:, 2]))
        vol[i] = float(np.sum(np.diff(np.log(mr)) ** 2))
        rr[i] = float(np.log(mr[-1]) - np.log(mr[0]))
        rg[i] = float(np.log(mg[-1]) - np.log(mg[0]))
    feats = [f for f in ws_features if f in dense_real and f in dense_gen]

    def ws(idx):
        vals = [w1(dense_real[f][idx[idx < len(dense_real[f])]], dense_gen[f][idx[idx < len(dense_gen[f])]])
                for f in feats]
        vals = [v for v in vals if np.isfinite(v)]
        return float(np.mean(vals)) if vals else None

    def ic_ci(idx):
        a, b = rg[idx], rr[idx]
        ok = np.isfinite(a) & np.isfinite(b)
        a, b = a[ok], b[ok]
        if a.size <= 2:
            return [float("nan"), float("nan")]
        rng = np.random.default_rng(seed)
        vals = [s for s in (_spearman(a[j], b[j]) for j in (rng.integers(0, a.size, a.size) for _ in range(n_boot)))
                if np.isfinite(s)]
        return [float(np.percentile(vals, 2.5)), float(np.percentile(vals, 97.5))] if vals else [float("nan")] * 2

    out = {"n_windows": int(n), "dense_features_used": feats}
    for name, strat in (("spread", spread), ("volatility", vol)):
        lab = _tertiles(strat)
        block = {}
        for k, t in enumerate(("low", "mid", "high")):
            idx = np.where(lab == k)[0]
            block[t] = {"n": int(idx.size), "ws": ws(idx) if feats else None, "ic": _spearman(rg[idx], rr[idx]),
                        "ic_ci": ic_ci(idx)}
        ics = [block[t]["ic"] for t in ("low", "mid", "high") if np.isfinite(block[t]["ic"])]
        block["ic_robustness_spread"] = float(max(ics) - min(ics)) if ics else None
        out[name] = block
    return {"eval": "regime_stratified", "data": out}


# ---------------------------------------------------------------------------
# position in the generated window
# ---------------------------------------------------------------------------

def position_in_window(dense_real: Dict[str, np.ndarray], dense_gen: Dict[str, np.ndarray], bin_width: int = 25,
                       features: Sequence[str] = ("spread", "ask_volume", "bid_volume", "orderbook_imbalance"),
                       c: Optional[int] = None) -> Dict:
    feats = [f for f in features if f in dense_real and f in dense_gen]
    if not feats:
        return {"eval": "position_in_window", "status": "no dense features"}
    g_len = min(dense_gen[f].shape[1] for f in feats)
    n_bins = max(1, g_len // bin_width)
    edges = (np.arange(n_bins + 1) * bin_width).astype(int)
    edges[-1] = g_len
    centers = (edges[:-1] + edges[1:]) / 2.0
    per, per_pool = {}, {}
    acc = np.full((len(feats), n_bins), np.nan)
    acc_pool = np.full((len(feats), n_bins), np.nan)
    for fi, f in enumerate(feats):
        G, R = dense_gen[f], dense_real[f]
        Rpool = _pooled(R)
        for bi in range(n_bins):
            cols = slice(edges[bi], edges[bi + 1])
            gv = G[:, cols]
            acc[fi, bi] = w1(gv, R[:, cols])
            acc_pool[fi, bi] = w1(gv, Rpool)
        per[f] = [float(x) for x in acc[fi]]
        per_pool[f] = [float(x) for x in acc_pool[fi]]
    with np.errstate(all="ignore"):
        ws_tau = np.nanmean(acc, 0)
        ws_pool = np.nanmean(acc_pool, 0)
    fit = fit_power_curve(centers, ws_tau)
    return {"eval": "position_in_window", "c": c, "g": int(g_len), "n_bins": int(n_bins), "bin_width": int(bin_width),
            "tau_centers": [float(x) for x in centers],
            "ws_tau": [None if not np.isfinite(x) else float(x) for x in ws_tau],
            "ws_tau_pooled": [None if not np.isfinite(x) else float(x) for x in ws_pool],
            "per_feature_ws_tau": per, "per_feature_ws_tau_pooled": per_pool, "fit_single_c": fit}


def fit_power_curve(tau: np.ndarray, y: np.ndarray) -> Dict:
    """Least-squares fit of y = alpha + beta * tau^p (alpha, beta >= 0, 0.2 <= p <= 3)."""
    good = np.isfinite(y)
    if good.sum() < 3:
        return {"status": "not enough bins"}
    from scipy.optimize import curve_fit
    t, v = np.asarray(tau, dtype=np.float64)[good], np.asarray(y, dtype=np.float64)[good]
    model = lambda x, a, b, p: a + b * np.power(np.clip(x, 1e-6, None), p)
    try:
        popt, _ = curve_fit(model, t, v, p0=[max(v.min(), 0.0), max(v.max() - v.min(), 1e-3), 1.0],
                            bounds=([0, 0, 0.2], [np.inf, np.inf, 3.0]), maxfev=20000)
    except (RuntimeError, ValueError) as e:
        return {"status": f"fit failed ({type(e).__name__})"}
    return {"alpha": float(popt[0]), "beta": float(popt[1]), "p": float(popt[2]),
            "model": "WS_tau = alpha + beta * tau^p (matched bins, tau in messages)"}


def fit_cg_surface(position_results: Sequence[Dict]) -> Dict:
    rows = sorted((float(r["c"]), r["fit_single_c"]["alpha"]) for r in position_results
                  if r.get("c") is not None and "alpha" in r.get("fit_single_c", {}))
    if len(rows) < 2:
        return {"status": "need >= 2 conditioning lengths with a fitted alpha"}
    cs = np.array([r[0] for r in rows])
    al = np.array([r[1] for r in rows])
    a0, amax = float(al[0]), float(al[-1])
    cstar = None
    if abs(a0 - amax) > 1e-12:
        below = cs[(al - amax) / (a0 - amax) < 0.1]
        cstar = float(below.min()) if below.size else None
    return {"alpha_of_c": {str(int(c)): float(a) for c, a in zip(cs, al)}, "alpha_0": a0, "alpha_cmax": amax,
            "c_star": cstar}


def run_all(msgs_real: Sequence[np.ndarray], books_real: Sequence[np.ndarray], msgs_gen: Sequence[np.ndarray],
            books_gen: Sequence[np.ndarray], bin_width: int = 25, c: Optional[int] = None) -> Dict[str, Dict]:
    """All three breakdowns from paired real / generated windows (messages + books)."""
    fr = [dense_features(m, b) for m, b in zip(msgs_real, books_real)]
    fg = [dense_features(m, b) for m, b in zip(msgs_gen, books_gen)]
    L = min([len(next(iter(w.values()))) for w in fr + fg] or [0])
    dr, dg = stack_windows(fr, L), stack_windows(fg, L)
    return {"tail": tail_conditioned(dr, dg), "regime": regime_stratified(books_real, books_gen, dr, dg),
            "position": position_in_window(dr, dg, bin_width=bin_width, c=c)}
