"""Observational comparisons of generated and real order flow: the joint volatility-volume
relation, the mid response to new limit orders by distance, resampler baselines and
run-to-run reproducibility.

The remaining analyse-only evaluations of the reference's
``tools/diagnostics/lob_evals.py`` (``eval_joint_canonical`` :508,
``eval_otm_observational`` :565, ``eval_baselines`` :726, ``eval_reproducibility`` :640),
written here over plain arrays (messages ``[time_s, time_ns, type, oid, size, price,
direction]``, L2 books ``[ask_p, ask_v, bid_p, bid_v, ...]``), with the reference's result
keys:

* ``joint_canonical`` -- per window, realised volatility (sum of squared log mid returns)
  and executed volume (sum of sizes of execution events); the Spearman correlation of the
  two across windows on each side, the difference with a bootstrap interval, the sliced
  2-Wasserstein distance between the jointly standardised (vol, volume) clouds, and the
  same distance between two halves of the real windows as the noise floor;
* ``otm_observational`` -- R(k): mean |mid(t + H) - mid(t)| in ticks after a new limit order
  placed k ticks from the mid, over a contiguous partition of k;
* ``resampler_baseline`` -- per feature, W1(real, generated) against W1(real, an i.i.d.
  resample of real of the generated size) and the gap closure
  (W1_resampler - W1_model) / W1_resampler (below 0: worse than resampling the marginal);
* ``reproducibility`` -- per feature, this run's W1 beside a baseline run's.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import numpy as np

from .conditioned import w1

EXEC = 4
LIMIT = 1
OTM_BINS = ((0, 5), (5, 15), (15, 35), (35, 75), (75, 150), (150, 500), (500, 1500), (1500, 10 ** 9))


def _mid(book: np.ndarray) -> np.ndarray:
    b = np.asarray(book, dtype=np.float64)
    return (b[:, 0] + b[:, 2]) / 2.0


def _spearman(x: np.ndarray, y: np.ndarray) -> float:
    from scipy.stats import spearmanr
    ok = np.isfinite(x) & np.isfinite(y) & (y > 0)
    return float(spearmanr(x[ok], y[ok]).statistic) if ok.sum() > 2 else float("nan")


def sliced_w2(X: np.ndarray, Y: np.ndarray, n_dirs: int = 50, seed: int = 0) -> float:
    """Sliced 2-Wasserstein distance between two point clouds: the root mean over random
    unit directions of the squared 1-D W2 between the projections (quantile matching)."""
    rng = np.random.default_rng(seed)
    vals = []
    for _ in range(n_dirs):
        th = rng.standard_normal(X.shape[1])
        th /= np.linalg.norm(th) + 1e-12
        xp, yp = np.sort(X @ th), np.sort(Y @ th)
        m = min(len(xp), len(yp))
        if m == 0:
            continue
        u = (np.arange(m) + 0.5) / m
        vals.append(np.mean((np.quantile(xp, u) - np.quantile(yp, u)) ** 2))
    return float(np.sqrt(np.mean(vals))) if vals else float("nan")


def _standardise_jointly(A: np.ndarray, B: np.ndarray):
    P = np.vstack([A, B])
    mu, sd = P.mean(0), P.std(0) + 1e-12
    return (A - mu) / sd, (B - mu) / sd


def _vol_volume(msgs: Sequence[np.ndarray], books: Sequence[np.ndarray]):
    sig, vol, nex = [], [], []
    for m, b in zip(msgs, books):
        m = np.asarray(m, dtype=np.float64)
        mid = np.clip(_mid(b), 1e-9, None)
        sig.append(float(np.sum(np.diff(np.log(mid)) ** 2)) if len(mid) > 1 else float("nan"))
        ex = m[:, 2] == EXEC
        vol.append(float(m[ex, 4].sum()))
        nex.append(int(ex.sum()))
    return np.array(sig), np.array(vol), np.array(nex)


def joint_canonical(msgs_real, books_real, msgs_gen, books_gen, n_boot: int = 200, seed: int = 0) -> Dict:
    sr, vr, nr = _vol_volume(msgs_real, books_real)
    sg, vg, ng = _vol_volume(msgs_gen, books_gen)
    rr, rg = _spearman(sr, vr), _spearman(sg, vg)
    rng = np.random.default_rng(seed)
    lo = hi = float("nan")
    if len(sr) > 2 and len(sg) > 2:
        d = np.array([_spearman(sg[j], vg[j]) - _spearman(sr[i], vr[i])
                      for i, j in ((rng.integers(0, len(sr), len(sr)), rng.integers(0, len(sg), len(sg)))
                                   for _ in range(n_boot))])
        if np.isfinite(d).any():
            lo, hi = np.nanpercentile(d, [2.5, 97.5])

    def cloud(s, v):
        ok = np.isfinite(s) & np.isfinite(v) & (v > 0)
        return np.column_stack([s[ok], v[ok]])
    Xr, Xg = cloud(sr, vr), cloud(sg, vg)
    sw2 = floor = float("nan")
    if len(Xr) > 4 and len(Xg) > 4:
        sw2 = sliced_w2(*_standardise_jointly(Xr, Xg), seed=seed)
        perm = rng.permutation(len(Xr))
        half = len(Xr) // 2
        floor = sliced_w2(*_standardise_jointly(Xr[perm[:half]], Xr[perm[half:2 * half]]), seed=seed)
    ok = np.isfinite(rr) and np.isfinite(rg)
    return {"eval": "joint_canonical", "rho_real": rr, "rho_gen": rg, "delta_rho": (rg - rr) if ok else None,
            "delta_rho_ci": [float(lo), float(hi)], "sliced_w2": sw2, "sliced_w2_floor_real_vs_real": floor,
            "closure": (1 - abs(rr - rg) / abs(rr)) if ok and abs(rr) > 1e-9 else None,
            "n_windows_real": int(len(sr)), "n_windows_gen": int(len(sg)),
            "exec_sparsity": {"mean_exec_per_window_real": float(nr.mean()) if nr.size else None,
                              "mean_exec_per_window_gen": float(ng.mean()) if ng.size else None,
                              "windows_with_zero_exec_real": int((nr == 0).sum()),
                              "windows_with_zero_exec_gen": int((ng == 0).sum())}}


def _response(msgs, books, H: int, tick: float):
    acc = {b: [] for b in OTM_BINS}
    for m, b in zip(msgs, books):
        m = np.asarray(m, dtype=np.float64)
        mid = _mid(b)
        new = np.where(m[:, 2] == LIMIT)[0]
        new = new[new + H < len(mid)]
        if new.size == 0:
            continue
        k = np.abs(m[new, 5] - mid[new]) / tick
        dmid = np.abs(mid[new + H] - mid[new]) / tick
        for lo, hi in OTM_BINS:
            sel = (k >= lo) & (k < hi)
            if sel.any():
                acc[(lo, hi)].extend(dmid[sel].tolist())
    return {f"{lo}-{hi}": (float(np.mean(v)) if v else None, len(v)) for (lo, hi), v in acc.items()}


def otm_observational(msgs_real, books_real, msgs_gen, books_gen, H: int = 100, tick: float = 100.0) -> Dict:
    return {"eval": "otm_observational", "H": H, "R_real": _response(msgs_real, books_real, H, tick),
            "R_gen": _response(msgs_gen, books_gen, H, tick)}


def resampler_baseline(real: Dict[str, np.ndarray], gen: Dict[str, np.ndarray], seed: int = 0) -> Dict:
    rng = np.random.default_rng(seed)
    res = {}
    for f in real:
        if f not in gen:
            continue
        r = np.asarray(real[f], dtype=np.float64).ravel()
        g = np.asarray(gen[f], dtype=np.float64).ravel()
        r, g = r[np.isfinite(r)], g[np.isfinite(g)]
        if r.size == 0 or g.size == 0:
            continue
        ws_model = w1(r, g)
        ws_res = w1(r, rng.choice(r, size=min(len(g), len(r)), replace=True))
        res[f] = {"ws_model": ws_model, "ws_resampler": ws_res,
                  "gap_closure": (ws_res - ws_model) / ws_res if ws_res > 1e-12 else None}
    return {"eval": "baselines", "resampler_gap_closure": res}


def reproducibility(this: Dict[str, float], baseline: Optional[Dict[str, float]]) -> Dict:
    """Per-feature W1 of this run beside a baseline run's ({feature: W1} each)."""
    if not baseline:
        return {"eval": "reproducibility", "status": "no baseline available"}
    return {"eval": "reproducibility",
            "per_feature": {f: {"this": float(v), "baseline": float(baseline[f])} for f, v in this.items()
                            if f in baseline}}
