"""Observational evaluations of generated order flow, stamped with provenance.

The analyse-only diagnostics of the reference's ``tools/diagnostics/lob_evals.py``
(own implementation, a subset): they read a finished generation run
(``data_gen/ data_real/`` CSVs, ``pipeline.lobbench.load_run``) and never generate.

* ``assert_generation_sane`` -- the sanity gate: refuse to report anything when the
  generated touch spreads fall far outside the real ones (a corrupted decode, e.g. an
  encoding mismatch, shows up there first);
* ``stylized_facts`` -- per side (real / generated): autocorrelation of mid returns
  (lag 1), of absolute returns at several lags (volatility clustering), the Hill tail
  index of |returns|, the leverage correlation corr(r_t, r_{t+k}^2), and the real -
  generated differences;
* ``tstr`` -- train on synthetic, test on real: a logistic model predicting the sign
  of the mid move over the next ``H`` events from order-flow imbalance features is
  fitted on generated windows and on real windows and both are scored by AUC on held-out
  real windows; the ratio (synthetic / real AUC excess over 0.5) is the headline;
* ``build_origin`` / ``stamp`` / ``write_provenance`` -- every number carries where it
  came from (run directory, checkpoint, experiment, ticker, depth);
* the tail-, regime- and position-conditioned breakdowns (``eval/conditioned.py``) and the
  joint volatility-volume, limit-order response, resampler-baseline and reproducibility
  comparisons (``eval/observational.py``), selected with ``--evals``.

    python -m sigma0_b200.eval.stylized --run <save_dir> --out <dir> [--experiment NAME]
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

EMPTY_PRICE = 2_147_483_647


def _touch(book: np.ndarray):
    b = np.asarray(book, dtype=np.float64)
    ask, bid = b[:, 0], b[:, 2]
    ok = (np.abs(ask) < EMPTY_PRICE) & (np.abs(bid) < EMPTY_PRICE) & (ask > 0) & (bid > 0)
    return ask, bid, ok


def _spreads(books: Sequence[np.ndarray]) -> np.ndarray:
    out = []
    for b in books:
        ask, bid, ok = _touch(b)
        out.append((ask - bid)[ok])
    return np.concatenate(out) if out else np.zeros(0)


def _mid_returns(book: np.ndarray) -> np.ndarray:
    ask, bid, ok = _touch(book)
    mid = 0.5 * (ask + bid)[ok]
    mid = mid[mid > 0]
    return np.diff(np.log(mid)) if len(mid) > 1 else np.zeros(0)


def build_origin(run_dir: str, experiment: str = "", ticker: str = "", depth: Optional[int] = None,
                 checkpoint: str = "", checkpoint_step: Optional[int] = None) -> Dict:
    return {"experiment": experiment, "ticker": ticker, "depth": depth, "run_dir": os.path.abspath(run_dir),
            "checkpoint": checkpoint, "checkpoint_step": checkpoint_step,
            "job_id": os.environ.get("SLURM_JOB_ID") or os.environ.get("JOB_ID", "")}


def stamp(result: Dict, origin: Dict) -> Dict:
    out = dict(result)
    out["origin"] = origin
    return out


def write_provenance(out_dir: str, origin: Dict, extra: Optional[Dict] = None) -> str:
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, "_provenance.json")
    with open(path, "w") as f:
        json.dump({"origin": origin, **(extra or {})}, f, indent=1, default=str)
    return path


class GenerationCorrupt(RuntimeError):
    pass


def assert_generation_sane(books_real: Sequence[np.ndarray], books_gen: Sequence[np.ndarray], origin: Dict,
                           factor: float = 20.0, max_bad_frac: float = 0.05) -> Dict:
    """Raise GenerationCorrupt when more than ``max_bad_frac`` of the generated spreads lie
    outside [min real / factor, max real * factor] (or there are none)."""
    sr, sg = _spreads(books_real), _spreads(books_gen)
    if len(sr) == 0:
        raise GenerationCorrupt(f"no valid real spreads in {origin.get('run_dir')}")
    lo, hi = max(sr.min() / factor, 0.0), sr.max() * factor
    bad = float(np.mean((sg < lo) | (sg > hi))) if len(sg) else 1.0
    info = {"real_spread_p50": float(np.median(sr)), "gen_spread_p50": float(np.median(sg)) if len(sg) else None,
            "bad_fraction": bad, "band": [float(lo), float(hi)]}
    if bad > max_bad_frac:
        raise GenerationCorrupt(f"generated spreads outside the real band in {bad:.1%} of frames: {info}")
    return info


def _acf(xs: List[np.ndarray], lag: int) -> float:
    num = den = 0.0
    allx = np.concatenate([x for x in xs if len(x)]) if any(len(x) for x in xs) else np.zeros(1)
    mu = allx.mean()
    for x in xs:
        if len(x) > lag:
            d = x - mu
            num += float(np.dot(d[:-lag], d[lag:]))
            den += float(np.dot(d, d))
    return num / den if den > 0 else float("nan")


def hill_index(x: np.ndarray, frac: float = 0.05) -> float:
    """Hill estimator of the tail index from the largest ``frac`` of |x|."""
    a = np.sort(np.abs(x[x != 0]))[::-1]
    k = max(int(len(a) * frac), 2)
    if len(a) <= k:
        return float("nan")
    return float(1.0 / np.mean(np.log(a[:k] / a[k])))


def stylized_facts(books_real: Sequence[np.ndarray], books_gen: Sequence[np.ndarray],
                   lags: Sequence[int] = (1, 5, 20)) -> Dict:
    out = {}
    for name, books in (("real", books_real), ("gen", books_gen)):
        r = [_mid_returns(b) for b in books]
        allr = np.concatenate([x for x in r if len(x)]) if any(len(x) for x in r) else np.zeros(0)
        d = {"ret_acf1": _acf(r, 1),
             **{f"absret_acf{k}": _acf([np.abs(x) for x in r], k) for k in lags},
             "hill_tail_index": hill_index(allr) if len(allr) > 10 else float("nan")}
        num = den = 0.0
        for x in r:
            if len(x) > 5:
                num += float(np.dot(x[:-5], x[5:] ** 2))
                den += float(np.sqrt(np.dot(x[:-5], x[:-5]) * np.dot(x[5:] ** 2, x[5:] ** 2)))
        d["leverage5"] = num / den if den > 0 else float("nan")
        out[name] = d
    out["diff"] = {k: out["real"][k] - out["gen"][k] for k in out["real"]}
    return out


def _ofi_features(msgs: np.ndarray, book: np.ndarray, H: int, W: int):
    """(features, labels): signed order flow over the last W events, spread and touch
    imbalance, and the sign of the mid move over the next H events, at every event with a
    valid book."""
    ask, bid, ok = _touch(book)
    b = np.asarray(book, dtype=np.float64)
    av, bv = b[:, 1], b[:, 3]
    mid = 0.5 * (ask + bid)
    side = np.where(np.asarray(msgs)[:, 6] > 0, 1.0, -1.0)
    size = np.asarray(msgs)[:, 4].astype(np.float64)
    etype = np.asarray(msgs)[:, 2]
    flow = np.where(etype == 1, side * size, np.where(etype == 4, -side * size, -side * size * (etype != 0)))
    cs = np.concatenate([[0.0], np.cumsum(flow)])
    X, y = [], []
    for t in range(W, len(mid) - H):
        if ok[t] and ok[t + H] and mid[t + H] != mid[t]:
            imb = (bv[t] - av[t]) / max(av[t] + bv[t], 1e-12)
            X.append([cs[t + 1] - cs[t + 1 - W], ask[t] - bid[t], imb])
            y.append(1.0 if mid[t + H] > mid[t] else 0.0)
    return np.array(X).reshape(-1, 3), np.array(y)


def _logistic(X, y, l2=1e-3, iters=200):
    mu, sd = X.mean(0), X.std(0) + 1e-9
    Z = np.c_[(X - mu) / sd, np.ones(len(X))]
    w = np.zeros(Z.shape[1])
    for _ in range(iters):                                  # Newton steps
        p = 1 / (1 + np.exp(-Z @ w))
        g = Z.T @ (p - y) + l2 * w
        Hm = (Z * (p * (1 - p))[:, None]).T @ Z + l2 * np.eye(len(w))
        w -= np.linalg.solve(Hm, g)
    return lambda Xn: 1 / (1 + np.exp(-np.c_[(Xn - mu) / sd, np.ones(len(Xn))] @ w))


def auc(scores: np.ndarray, y: np.ndarray) -> float:
    """Area under the ROC curve (rank statistic, ties averaged)."""
    from scipy.stats import rankdata
    pos, n1 = y == 1, int((y == 1).sum())
    n0 = len(y) - n1
    if n1 == 0 or n0 == 0:
        return float("nan")
    r = rankdata(scores)
    return float((r[pos].sum() - n1 * (n1 + 1) / 2) / (n1 * n0))


def tstr(msgs_real, books_real, msgs_gen, books_gen, H: int = 10, W: int = 20, seed: int = 0,
         n_boot: int = 200) -> Dict:
    """Train on synthetic, test on real: a mid-direction predictor on [windowed OFI, spread,
    touch imbalance] fitted on generated windows (s -> r) and on real training windows
    (r -> r), both scored by AUC on the same held-out real windows.  Reports the AUC ratio
    s->r / r->r with a bootstrap interval over test windows, the excess-over-chance ratio,
    and a gradient-boosting row when scikit-learn is installed."""
    rng = np.random.default_rng(seed)
    n = len(books_real)
    perm = rng.permutation(n)
    test, train = perm[: max(n // 3, 1)], perm[max(n // 3, 1):]

    def feats(ms, bs, idx):
        parts = [(_ofi_features(ms[i], bs[i], H, W), i) for i in idx]
        X = np.concatenate([p[0][0] for p in parts]) if parts else np.zeros((0, 3))
        y = np.concatenate([p[0][1] for p in parts]) if parts else np.zeros(0)
        wid = np.concatenate([np.full(len(p[0][1]), p[1]) for p in parts]) if parts else np.zeros(0)
        return X, y, wid
    Xte, yte, wte = feats(msgs_real, books_real, test)
    Xr, yr, _ = feats(msgs_real, books_real, train)
    Xg, yg, _ = feats(msgs_gen, books_gen, range(len(books_gen)))
    res = {"n_test": int(len(yte)), "n_train_real": int(len(yr)), "n_train_gen": int(len(yg)),
           "n_test_windows": int(len(np.unique(wte)))}
    if min(len(yte), len(yr), len(yg)) < 10 or len(set(yr)) < 2 or len(set(yg)) < 2 or len(set(yte)) < 2:
        res["skipped"] = "too few labelled events"
        return res
    pr, pg = _logistic(Xr, yr)(Xte), _logistic(Xg, yg)(Xte)
    res["auc_trained_on_real"] = auc(pr, yte)
    res["auc_trained_on_gen"] = auc(pg, yte)
    ex_r = res["auc_trained_on_real"] - 0.5
    res["tstr_ratio"] = (res["auc_trained_on_gen"] - 0.5) / ex_r if abs(ex_r) > 1e-9 else float("nan")
    a_rr = res["auc_trained_on_real"]
    res["auc_ratio"] = res["auc_trained_on_gen"] / a_rr if a_rr > 0 else float("nan")
    rows = {w: np.where(wte == w)[0] for w in np.unique(wte)}
    ws = list(rows)
    ratios = []
    for _ in range(n_boot):
        sel = np.concatenate([rows[ws[i]] for i in rng.integers(0, len(ws), len(ws))])
        if len(set(yte[sel])) < 2:
            continue
        rr_ = auc(pr[sel], yte[sel])
        if rr_ > 0:
            ratios.append(auc(pg[sel], yte[sel]) / rr_)
    res["auc_ratio_ci"] = ([float(np.percentile(ratios, 2.5)), float(np.percentile(ratios, 97.5))]
                          if ratios else [float("nan")] * 2)
    try:
        from sklearn.ensemble import HistGradientBoostingClassifier

        def gbm(X, y):
            m = HistGradientBoostingClassifier(max_depth=3, max_iter=120, learning_rate=0.08, random_state=0)
            m.fit(X, y)
            return auc(m.predict_proba(Xte)[:, 1], yte)
        g_rr, g_sr = gbm(Xr, yr), gbm(Xg, yg)
        res["gbm"] = {"auc_rr": g_rr, "auc_sr": g_sr, "ratio": g_sr / g_rr if g_rr > 0 else float("nan")}
    except ImportError:
        res["gbm"] = {"status": "skipped (scikit-learn not installed)"}
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--run", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--experiment", default="")
    ap.add_argument("--ticker", default="")
    ap.add_argument("--checkpoint", default="")
    ALL = ["stylized", "tstr", "tail", "regime", "position", "joint", "otm", "baselines", "repro"]
    ap.add_argument("--evals", nargs="+", default=ALL, choices=ALL)
    ap.add_argument("--baseline", default="", help="repro: a previous diagnostics output directory")
    ap.add_argument("--otm_h", type=int, default=100, help="otm: horizon in messages")
    ap.add_argument("--bin_width", type=int, default=25, help="position-in-window bin width (messages)")
    ap.add_argument("--cond_msgs", type=int, default=None, help="conditioning length c of the run (position eval)")
    a = ap.parse_args(argv)
    from ..pipeline.lobbench import load_run
    run = load_run(a.run)
    ids = sorted(i for i, d in run.items() if "gen" in d and "real" in d)
    mr = [run[i]["real"][0] for i in ids]
    br = [run[i]["real"][1][:, 3:] if run[i]["real"][1].shape[1] % 4 == 3 else run[i]["real"][1] for i in ids]
    mg = [run[i]["gen"][0] for i in ids]
    bg = [run[i]["gen"][1][:, 3:] if run[i]["gen"][1].shape[1] % 4 == 3 else run[i]["gen"][1] for i in ids]
    depth = br[0].shape[1] // 4 if br else None
    origin = build_origin(a.run, a.experiment, a.ticker, depth, a.checkpoint)
    write_provenance(a.out, origin, {"windows": len(ids)})
    results = {"sanity": assert_generation_sane(br, bg, origin)}
    if "stylized" in a.evals:
        results["stylized_facts"] = stylized_facts(br, bg)
    if "tstr" in a.evals:
        results["tstr"] = tstr(mr, br, mg, bg)
    cond = [e for e in ("tail", "regime", "position") if e in a.evals]
    if cond:
        from .conditioned import run_all
        res = run_all(mr, br, mg, bg, bin_width=a.bin_width, c=a.cond_msgs)
        for e in cond:
            results[e] = res[e]
    from . import observational as O
    if "joint" in a.evals:
        results["joint"] = O.joint_canonical(mr, br, mg, bg)
    if "otm" in a.evals:
        results["otm"] = O.otm_observational(mr, br, mg, bg, H=a.otm_h)
    if "baselines" in a.evals or "repro" in a.evals:
        from .conditioned import dense_features, w1
        fr = [dense_features(m, b) for m, b in zip(mr, br)]
        fg = [dense_features(m, b) for m, b in zip(mg, bg)]
        pool = lambda fs, f: np.concatenate([w[f] for w in fs]) if fs else np.zeros(0)
        real = {f: pool(fr, f) for f in (fr[0] if fr else {})}
        gen = {f: pool(fg, f) for f in (fg[0] if fg else {})}
        if "baselines" in a.evals:
            results["baselines"] = O.resampler_baseline(real, gen)
        if "repro" in a.evals:
            this = {f: w1(real[f], gen[f]) for f in real if f in gen}
            base = None
            bp = os.path.join(a.baseline, "repro.json") if a.baseline else ""
            if bp and os.path.exists(bp):
                with open(bp) as fh:
                    base = {f: v["this"] for f, v in json.load(fh).get("per_feature", {}).items()}
            res = O.reproducibility(this, base)
            res.setdefault("per_feature", {f: {"this": v} for f, v in this.items()})
            results["repro"] = res
    for k, v in results.items():
        with open(os.path.join(a.out, f"{k}.json"), "w") as f:
            json.dump(stamp(v, origin), f, indent=1, default=float)
    big = ("tail", "regime", "position", "joint", "otm", "baselines", "repro")
    summary = {k: (v["diff"] if k == "stylized_facts" else v) for k, v in results.items() if k not in big}
    summary.update({k: "written" for k in big if k in results})
    print(json.dumps(summary, default=float))


if __name__ == "__main__":
    main()
