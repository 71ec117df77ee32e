"""Event-anchored return bench: does the generated continuation of a window predict the mid
price move that really followed?

The reference's bench (``src/lobpipeline/return_bench/event_anchored.py:66-306``,
``run_event_bench.py:61-335``) scores generation runs at wall-clock horizons after an anchor:
the window's last conditioning message, which must be a trade.  For every window and horizon
the generated stream's log return of the mid and the real stream's are paired; the skill
numbers are IC (Pearson), ranked IC (Spearman) and direction accuracy over samples whose
real return is not zero, next to their distribution under random re-pairing (the shuffle
null: direction accuracy under it is not 50% when real returns are not sign-balanced) and the
baseline that uses no model at all, the return sign the anchoring trade implies.  Rules kept
because each one changes answers without raising anything when broken:

* a horizon past the end of a stream is not covered -- the sample is dropped for that
  horizon, never answered with the stream's last row;
* the price at ``t0 + h`` is the mid after the LAST message at or before that time
  (messages sharing the target timestamp count; the one after it does not);
* no message at or before the target means the book is untouched: the anchor's mid;
* a horizon is scored only where both streams cover it;
* ``identity`` feeds the real stream in as the generated one, and IC must come out 1.

Streams are this package's engine rows (``sim.divergence.read_messages``: time in columns 6
and 7, direction in column 1) and L2 book rows after each message.
"""
from __future__ import annotations

import argparse
import json
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

ZERO_RETURN = 1e-12


def mids(books: np.ndarray) -> np.ndarray:
    """Mid per book row; NaN where either side of the touch is empty."""
    b = np.asarray(books, np.float64)
    ask, bid = b[:, 0], b[:, 2]
    m = (ask + bid) / 2.0
    m[(ask <= 0) | (bid <= 0) | (ask >= 2 ** 31 - 1)] = np.nan
    return m


def times_of(msgs: np.ndarray) -> np.ndarray:
    m = np.asarray(msgs, np.int64)
    return m[:, 6].astype(np.float64) + m[:, 7].astype(np.float64) * 1e-9


def price_at(times: np.ndarray, mid: np.ndarray, t0: float, p0: float, horizon_ms: float) -> Tuple[bool, float]:
    """(covered, mid as of t0 + horizon): the mid after the last message at or before the
    target; the anchor's mid if no message came by then; not covered past the stream's end."""
    times = np.asarray(times, np.float64)
    target = t0 + horizon_ms / 1000.0
    if times.size == 0 or times[-1] < target:
        return False, float("nan")
    j = int(np.searchsorted(times, target, side="right")) - 1
    return True, float(p0) if j < 0 else float(mid[j])


def anchored_returns(horizons_ms: Sequence[float], t0: float, p0: float, gen_times, gen_mid, real_times,
                     real_mid) -> Dict[float, Tuple[float, float]]:
    """{horizon: (generated log return, real log return)} where both streams cover it."""
    out: Dict[float, Tuple[float, float]] = {}
    if not np.isfinite(p0) or p0 <= 0:
        return out
    for h in horizons_ms:
        cg, pg = price_at(gen_times, gen_mid, t0, p0, h)
        cr, pr = price_at(real_times, real_mid, t0, p0, h)
        if cg and cr and np.isfinite(pg) and np.isfinite(pr) and pg > 0 and pr > 0:
            out[h] = (float(np.log(pg / p0)), float(np.log(pr / p0)))
    return out


def _rank(x: np.ndarray) -> np.ndarray:
    order = np.argsort(x, kind="stable")
    r = np.empty(len(x), np.float64)
    r[order] = np.arange(len(x), dtype=np.float64)
    # average ranks of ties
    xs = x[order]
    i = 0
    while i < len(xs):
        j = i
        while j + 1 < len(xs) and xs[j + 1] == xs[i]:
            j += 1
        if j > i:
            r[order[i:j + 1]] = (i + j) / 2.0
        i = j + 1
    return r


def _corr(a: np.ndarray, b: np.ndarray) -> float:
    a, b = a - a.mean(), b - b.mean()
    d = np.sqrt((a * a).sum() * (b * b).sum())
    return float((a * b).sum() / d) if d > 0 else float("nan")


def skill(pred: np.ndarray, real: np.ndarray) -> Dict[str, float]:
    """IC, ranked IC and direction accuracy (over samples with a non-zero real return)."""
    pred, real = np.asarray(pred, np.float64), np.asarray(real, np.float64)
    n = int(pred.size)
    if n < 3:
        return {"IC": float("nan"), "ranked_IC": float("nan"), "direction_acc": float("nan"), "N": n, "N_eff": 0}
    nz = np.abs(real) > ZERO_RETURN
    acc = float(np.mean(np.sign(pred[nz]) == np.sign(real[nz]))) if nz.any() else float("nan")
    return {"IC": _corr(pred, real), "ranked_IC": _corr(_rank(pred), _rank(real)), "direction_acc": acc,
            "N": n, "N_eff": int(nz.sum())}


def shuffle_null(pred: np.ndarray, real: np.ndarray, n_draws: int = 200, seed: int = 0) -> Dict[str, float]:
    """Mean and spread of the skill numbers under random re-pairing of the samples."""
    pred, real = np.asarray(pred, np.float64), np.asarray(real, np.float64)
    if pred.size < 5:
        return {"IC_mean": float("nan"), "IC_sd": float("nan"), "dir_acc_mean": float("nan")}
    rng = np.random.default_rng(seed)
    ics, accs = [], []
    for _ in range(n_draws):
        s = skill(pred[rng.permutation(pred.size)], real)
        ics.append(s["IC"])
        accs.append(s["direction_acc"])
    return {"IC_mean": float(np.nanmean(ics)), "IC_sd": float(np.nanstd(ics)),
            "dir_acc_mean": float(np.nanmean(accs))}


def trade_sign_baseline(directions) -> np.ndarray:
    """The move the anchoring trade implies on its own: a trade against a resting bid
    (direction +1) is seller-initiated, so the mid should fall."""
    return -np.asarray(directions, np.float64)


def magnitude_skill(pred: np.ndarray, real: np.ndarray) -> Dict[str, float]:
    """Does the generated move have the right size: correlation of |pred| with |real| and
    the ratio of their mean absolute values."""
    pred, real = np.abs(np.asarray(pred, np.float64)), np.abs(np.asarray(real, np.float64))
    if pred.size < 3:
        return {"abs_corr": float("nan"), "abs_ratio": float("nan")}
    return {"abs_corr": _corr(pred, real),
            "abs_ratio": float(pred.mean() / real.mean()) if real.mean() > 0 else float("nan")}


def clock_counts(gen_times, real_times, t0: float, horizon_ms: float) -> Tuple[int, int]:
    """Messages each stream put into (t0, t0 + horizon]: a millisecond horizon also scores the
    generator's clock, and diverging counts separate a clock problem from a price problem."""
    t1 = t0 + horizon_ms / 1000.0
    g, r = np.asarray(gen_times), np.asarray(real_times)
    return int(((g > t0) & (g <= t1)).sum()), int(((r > t0) & (r <= t1)).sum())


def bench(windows: Sequence[Dict], horizons_ms: Sequence[float], identity: bool = False,
          require_trade: bool = True, n_null: int = 200) -> Dict[str, Dict]:
    """Score windows ``{"cond_msgs", "cond_books", "real_msgs", "real_books", "gen_msgs",
    "gen_books"}`` (engine rows and book rows after each message); per horizon the skill
    numbers, the shuffle null, the trade-sign baseline, magnitude skill and message counts."""
    per: Dict[float, List] = {h: [] for h in horizons_ms}
    dirs: Dict[float, List[float]] = {h: [] for h in horizons_ms}
    counts: Dict[float, List[Tuple[int, int]]] = {h: [] for h in horizons_ms}
    used = 0
    for w in windows:
        cm = np.asarray(w["cond_msgs"], np.int64)
        if require_trade and int(cm[-1, 0]) != 4:
            continue
        used += 1
        t0 = float(times_of(cm[-1:])[0])
        p0 = float(mids(np.asarray(w["cond_books"])[-1:])[0])
        rt, rm = times_of(w["real_msgs"]), mids(w["real_books"])
        gt, gm = (rt, rm) if identity else (times_of(w["gen_msgs"]), mids(w["gen_books"]))
        for h, pair in anchored_returns(horizons_ms, t0, p0, gt, gm, rt, rm).items():
            per[h].append(pair)
            dirs[h].append(float(cm[-1, 1]))
            counts[h].append(clock_counts(gt, rt, t0, h))
    out = {"windows_used": used, "horizons": {}}
    for h in horizons_ms:
        if not per[h]:
            out["horizons"][str(h)] = {"N": 0}
            continue
        pred, real = np.array(per[h]).T
        c = np.array(counts[h])
        out["horizons"][str(h)] = {**skill(pred, real), "null": shuffle_null(pred, real, n_null),
                                   "trade_sign_baseline": skill(trade_sign_baseline(dirs[h]), real),
                                   **magnitude_skill(pred, real),
                                   "gen_msgs_mean": float(c[:, 0].mean()), "real_msgs_mean": float(c[:, 1].mean())}
    return out


def load_run(root: str, stock: str, limit: int = 10 ** 6) -> List[Dict]:
    """The windows of a generation run (``cli/infer.py`` layout)."""
    from ..sim.divergence import read_books, read_messages, run_paths
    from ..sim.frozen import run_windows
    out = []
    for date, i in run_windows(root, stock, limit):
        p = run_paths(root, stock, date, i)
        out.append({"window": f"{date} #{i}", "cond_msgs": read_messages(p["cond_msg"]),
                    "cond_books": read_books(p["cond_book"]), "real_msgs": read_messages(p["real_msg"]),
                    "real_books": read_books(p["real_book"]), "gen_msgs": read_messages(p["gen_msg"]),
                    "gen_books": read_books(p["gen_book"])})
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--run_dir", required=True)
    ap.add_argument("--stock", default="SYN")
    ap.add_argument("--horizons_ms", type=float, nargs="+", default=[10, 50, 100, 500])
    ap.add_argument("--identity_check", action="store_true",
                    help="score the real continuation as if generated: IC must be exactly 1")
    ap.add_argument("--any_anchor", action="store_true", help="do not require the last conditioning message to be a trade")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    res = bench(load_run(a.run_dir, a.stock), a.horizons_ms, a.identity_check, not a.any_anchor)
    text = json.dumps(res, indent=1)
    print(text)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    if a.identity_check:
        ics = [v.get("IC") for v in res["horizons"].values() if v.get("N", 0) >= 3]
        if not ics or any(not np.isfinite(x) or abs(x - 1.0) > 1e-12 for x in ics):
            return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
