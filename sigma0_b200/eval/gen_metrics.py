"""Per-step metrics of generated continuations against the real ones (the reference's
generator evaluation, ``src/base_model/inference/evaluation.py:14-430``).

* book losses between a generated and a real L2 snapshot, compared by price, not by level:
  each book becomes a signed volume profile over prices (asks negative, bids positive), both
  are put on the union of their prices, and only prices inside the range spanned by the
  first ``n_levels`` levels of either book count.  ``book_loss_l1`` is the summed absolute
  volume difference divided by the number of prices compared; ``book_loss_wasserstein`` the
  1-Wasserstein distance between the two profiles, each normalised to unit absolute mass
  (the cumulative difference summed along the price axis);
* ``mid_loss_l1``: |generated mid - real mid| in ticks; ``return_sq_err``: squared
  difference of the two returns from a common start mid;
* ``return_corr`` across windows per step, with a bootstrap interval;
* ``moments`` (mean, std, skew, excess kurtosis) of returns with bootstrap intervals;
* ``liquidity``: cumulative volume of new orders (provided) and of cancels / executions
  (taken) along a message stream; ``event_type_counts``.

Books are rows ``[ask_p, ask_v, bid_p, bid_v] x levels`` (empty levels at the engine's
sentinel prices or non-positive); messages the package's 14-column rows (event type in
column 1, size in column 5) or engine rows (type 0, size 2).

``python -m sigma0_b200.eval.gen_metrics --run_dir RUN --stock SYN`` scores a generation run
(``cli/infer.py`` layout) over the windows' common number of generated steps.
"""
from __future__ import annotations

from typing import Callable, Dict, Tuple

import numpy as np

EMPTY_ASK = 2 ** 31 - 1


def _profile(row: np.ndarray) -> Dict[int, float]:
    """price -> signed volume (asks negative) of one L2 row."""
    r = np.asarray(row, np.int64).reshape(-1, 4)
    out: Dict[int, float] = {}
    for ap, av, bp, bv in r:
        if 0 < ap < EMPTY_ASK:
            out[int(ap)] = out.get(int(ap), 0.0) - float(av)
        if bp > 0:
            out[int(bp)] = out.get(int(bp), 0.0) + float(bv)
    return out


def _price_range(row: np.ndarray, n_levels: int) -> Tuple[float, float]:
    r = np.asarray(row, np.int64).reshape(-1, 4)[:n_levels]
    ps = [p for p in np.concatenate([r[:, 0], r[:, 2]]) if 0 < p < EMPTY_ASK]
    return (min(ps), max(ps)) if ps else (np.inf, -np.inf)


def compared_volumes(gen: np.ndarray, real: np.ndarray, n_levels: int) -> Tuple[np.ndarray, np.ndarray]:
    """The two signed volume profiles on the union of their prices inside the compared range
    (sorted by price)."""
    pg, pr = _profile(gen), _profile(real)
    lo_g, hi_g = _price_range(gen, n_levels)
    lo_r, hi_r = _price_range(real, n_levels)
    lo, hi = min(lo_g, lo_r), max(hi_g, hi_r)
    prices = sorted(p for p in set(pg) | set(pr) if lo <= p <= hi)
    return (np.array([pg.get(p, 0.0) for p in prices]), np.array([pr.get(p, 0.0) for p in prices]))


def book_loss_l1(gen: np.ndarray, real: np.ndarray, n_levels: int = 10) -> float:
    vg, vr = compared_volumes(gen, real, n_levels)
    return float(np.abs(vg - vr).sum() / len(vg)) if len(vg) else float("nan")


def book_loss_wasserstein(gen: np.ndarray, real: np.ndarray, n_levels: int = 10) -> float:
    vg, vr = compared_volumes(gen, real, n_levels)
    if not len(vg) or not np.abs(vg).sum() or not np.abs(vr).sum():
        return float("nan")
    d = vg / np.abs(vg).sum() - vr / np.abs(vr).sum()
    return float(np.abs(np.cumsum(d)).sum())


def _mid(books: np.ndarray) -> np.ndarray:
    b = np.asarray(books, np.float64)
    return (b[..., 0] + b[..., 2]) / 2.0


def mid_loss_l1(gen_books: np.ndarray, real_books: np.ndarray, tick: int = 100) -> np.ndarray:
    """Per step |generated mid - real mid| in ticks."""
    return np.abs(_mid(gen_books) - _mid(real_books)) / tick


def return_sq_err(gen_mid: np.ndarray, real_mid: np.ndarray, mid0) -> np.ndarray:
    mid0 = np.asarray(mid0, np.float64)
    return np.square((np.asarray(gen_mid) - mid0) / mid0 - (np.asarray(real_mid) - mid0) / mid0)


def bootstrap_ci(x: np.ndarray, stat: Callable[[np.ndarray], float], n_boot: int = 1000, ci: float = 0.95,
                 seed: int = 0) -> Tuple[float, float]:
    """Percentile interval of ``stat`` over resamples of the rows of ``x``."""
    x = np.asarray(x)
    rng = np.random.default_rng(seed)
    vals = [stat(x[rng.integers(0, len(x), len(x))]) for _ in range(n_boot)]
    a = (1.0 - ci) / 2.0
    return float(np.nanquantile(vals, a)), float(np.nanquantile(vals, 1.0 - a))


def return_corr(rets_gen: np.ndarray, rets_real: np.ndarray) -> np.ndarray:
    """Correlation across windows of generated and real returns, per step (columns)."""
    g, r = np.asarray(rets_gen, np.float64), np.asarray(rets_real, np.float64)
    g, r = g - g.mean(0), r - r.mean(0)
    den = np.sqrt((g * g).sum(0) * (r * r).sum(0))
    with np.errstate(invalid="ignore", divide="ignore"):
        return np.where(den > 0, (g * r).sum(0) / den, np.nan)


def return_corr_ci(rets_gen: np.ndarray, rets_real: np.ndarray, n_boot: int = 500, ci: float = 0.95,
                   seed: int = 0) -> Tuple[np.ndarray, np.ndarray]:
    """Per-step bootstrap interval of ``return_corr`` (windows resampled together)."""
    g, r = np.asarray(rets_gen, np.float64), np.asarray(rets_real, np.float64)
    rng = np.random.default_rng(seed)
    vals = []
    for _ in range(n_boot):
        i = rng.integers(0, len(g), len(g))
        vals.append(return_corr(g[i], r[i]))
    vals = np.array(vals)
    a = (1.0 - ci) / 2.0
    return np.nanquantile(vals, a, axis=0), np.nanquantile(vals, 1.0 - a, axis=0)


def moments(rets: np.ndarray) -> Dict[str, float]:
    x = np.asarray(rets, np.float64).ravel()
    m, s = x.mean(), x.std()
    z = (x - m) / s if s > 0 else np.zeros_like(x)
    return {"mean": float(m), "std": float(s), "skew": float((z ** 3).mean()),
            "excess_kurtosis": float((z ** 4).mean() - 3.0)}


def moments_ci(rets: np.ndarray, n_boot: int = 500, ci: float = 0.95, seed: int = 0) -> Dict[str, Tuple[float, float]]:
    x = np.asarray(rets, np.float64).ravel()
    return {k: bootstrap_ci(x, lambda y, k=k: moments(y)[k], n_boot, ci, seed) for k in moments(x)}


def _cols(m: np.ndarray) -> Tuple[int, int]:
    """(event type, size) columns: the 14-column message rows or the 8-column engine rows."""
    return (0, 2) if m.shape[-1] == 8 else (1, 5)


def liquidity(msgs: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Cumulative volume provided (new orders) and taken (cancels, deletes, executions)."""
    m = np.asarray(msgs, np.int64)
    te, sz = _cols(m)
    etype, size = m[..., te], m[..., sz]
    return np.cumsum(np.where(etype == 1, size, 0), -1), np.cumsum(np.where(etype > 1, size, 0), -1)


def event_type_counts(msgs: np.ndarray, types=(1, 2, 3, 4)) -> Dict[int, int]:
    m = np.asarray(msgs, np.int64)
    e = m[..., _cols(m)[0]].ravel()
    return {int(t): int((e == t).sum()) for t in types}


def evaluate(gen_books: np.ndarray, real_books: np.ndarray, gen_msgs: np.ndarray, real_msgs: np.ndarray,
             mid0: np.ndarray, n_levels: int = 10, tick: int = 100, n_boot: int = 200) -> Dict:
    """The whole set for W windows of S steps: books (W, S, 4L), messages (W, S, 14), start
    mids (W,).  Book losses against a constant-book baseline (the conditioning book held
    fixed) say how much the generator adds over predicting no change."""
    gb, rb = np.asarray(gen_books), np.asarray(real_books)
    W, S = gb.shape[:2]
    l1 = np.array([[book_loss_l1(gb[w, s], rb[w, s], n_levels) for s in range(S)] for w in range(W)])
    ws = np.array([[book_loss_wasserstein(gb[w, s], rb[w, s], n_levels) for s in range(S)] for w in range(W)])
    gm, rm = _mid(gb), _mid(rb)
    mid0 = np.asarray(mid0, np.float64)
    rg, rr = (gm - mid0[:, None]) / mid0[:, None], (rm - mid0[:, None]) / mid0[:, None]
    lo, hi = return_corr_ci(rg, rr, n_boot)
    return {"book_loss_l1": np.nanmean(l1, 0).tolist(), "book_loss_wasserstein": np.nanmean(ws, 0).tolist(),
            "mid_loss_l1_ticks": mid_loss_l1(gb, rb, tick).mean(0).tolist(),
            "return_sq_err": return_sq_err(gm, rm, mid0[:, None]).mean(0).tolist(),
            "return_corr": return_corr(rg, rr).tolist(), "return_corr_ci": [lo.tolist(), hi.tolist()],
            "moments_gen": moments(rg[:, -1]), "moments_real": moments(rr[:, -1]),
            "events_gen": event_type_counts(gen_msgs), "events_real": event_type_counts(real_msgs)}


def evaluate_run(root: str, stock: str, n_levels: int = 10, tick: int = 100, limit: int = 10 ** 6,
                 n_boot: int = 200) -> Dict:
    """``evaluate`` over the windows of a generation run, cut to their common length."""
    from ..sim.divergence import read_books, read_messages, run_paths
    from ..sim.frozen import run_windows
    gb, rb, gm, rm, m0 = [], [], [], [], []
    for date, i in run_windows(root, stock, limit):
        p = run_paths(root, stock, date, i)
        gb.append(read_books(p["gen_book"]))
        rb.append(read_books(p["real_book"]))
        gm.append(read_messages(p["gen_msg"]))
        rm.append(read_messages(p["real_msg"]))
        m0.append(float(_mid(read_books(p["cond_book"])[-1:])[0]))
    if not gb:
        raise FileNotFoundError(f"no generated windows under {root}/data_gen")
    S = min(min(len(x) for x in gb), min(len(x) for x in rb))
    w = min(b.shape[1] for b in gb + rb)
    cut = lambda xs, c=None: np.stack([x[:S, :c] if c else x[:S] for x in xs])
    res = evaluate(cut(gb, w), cut(rb, w), cut(gm), cut(rm), np.array(m0), n_levels, tick, n_boot)
    res.update(n_windows=len(gb), n_steps=S)
    return res


def main(argv=None) -> int:
    import argparse
    import json
    ap = argparse.ArgumentParser(description="generator metrics of a generation run against the real continuations")
    ap.add_argument("--run_dir", required=True)
    ap.add_argument("--stock", default="SYN")
    ap.add_argument("--n_levels", type=int, default=10)
    ap.add_argument("--tick", type=int, default=100)
    ap.add_argument("--n_boot", type=int, default=200)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    res = evaluate_run(a.run_dir, a.stock, a.n_levels, a.tick, n_boot=a.n_boot)
    text = json.dumps(res, indent=1)
    print(text)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
