"""LOB-Bench style scoring of a generation run directory.

Reads the ``data_cond/ data_gen/ data_real/`` CSV layout written by the
generation runtime and scores generated against real order flow with the
marginal statistics of ``eval/lob_metrics.py`` (W1 / KS / L1 with bootstrap
intervals).  Modes (the reference adapter's, ``lobpipeline/lob_bench/scoring.py``):

* ``uncond``       -- pooled marginals of all generated vs all real continuations;
* ``cond``         -- per window, generated vs its own real continuation, averaged;
* ``context``      -- the real conditioning window vs the real continuation (a
                      "nothing changes" baseline every model should beat);
* ``time_lagged``  -- real continuation of window i vs that of window i+1 (the
                      natural variability floor);
* ``divergence``   -- the ``cond`` distance per horizon bucket (how fast
                      generated paths drift from the real ones).

``shard`` / ``merge`` split a run's windows over workers and combine their JSON
summaries (weighted by window count).
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import re
from typing import Dict, List, Tuple

import numpy as np

from ..eval.lob_metrics import concat_marginals, marginals, score

_MSG = re.compile(r"^(?P<pre>.+)_message_real_id_(?P<i>\d+)(?P<gen>_gen_id_0)?\.csv$")


def _read_msgs(path: str) -> np.ndarray:
    import pandas as pd
    df = pd.read_csv(path, dtype={"time": str})
    t = df["time"].str.split(".", expand=True)
    return np.stack([t[0].astype(np.int64), t[1].str.pad(9, "right", "0").astype(np.int64), df["event_type"],
                     df["order_id"], df["size"], df["price"], df["direction"]], 1).astype(np.float64)


def _read_books(path: str) -> np.ndarray:
    import pandas as pd
    return pd.read_csv(path).to_numpy().astype(np.float64)


def load_run(save_dir: str) -> Dict[int, Dict[str, Tuple[np.ndarray, np.ndarray]]]:
    """{window: {"gen"|"real"|"cond": (msgs, books)}}"""
    out: Dict[int, Dict] = {}
    for sub, key in (("data_gen", "gen"), ("data_real", "real"), ("data_cond", "cond")):
        for p in glob.glob(os.path.join(save_dir, sub, "*_message_real_id_*.csv")):
            m = _MSG.match(os.path.basename(p))
            if not m:
                continue
            i = int(m["i"])
            bp = p.replace("_message_", "_orderbook_")
            books = _read_books(bp)
            msgs = _read_msgs(p)
            if key == "cond":
                books = books[1:]          # N+1 rows: drop the opening snapshot
            out.setdefault(i, {})[key] = (msgs, books[:len(msgs)])
    return out


def _summ(scores) -> Dict[str, Dict[str, float]]:
    return {s.metric: {"value": s.value, "ci_low": s.ci_low, "ci_high": s.ci_high} for s in scores}


def score_run(save_dir: str, mode: str = "uncond", n_boot: int = 50, buckets: int = 4,
              windows: List[int] = None) -> Dict:
    run = load_run(save_dir)
    ids = sorted(i for i in run if "gen" in run[i] and "real" in run[i])
    if windows is not None:
        ids = [i for i in ids if i in set(windows)]
    if not ids:
        raise FileNotFoundError(f"no scored windows under {save_dir}")
    res = {"mode": mode, "n_windows": len(ids)}
    if mode == "uncond":
        g = concat_marginals(marginals(*run[i]["gen"]) for i in ids)
        r = concat_marginals(marginals(*run[i]["real"]) for i in ids)
        res["scores"] = _summ(score(g, r, n_boot=n_boot))
    elif mode == "cond":
        per = [_summ(score(marginals(*run[i]["gen"]), marginals(*run[i]["real"]), n_boot=0)) for i in ids]
        res["scores"] = {}
        for k in per[0]:
            v = np.array([p[k]["value"] for p in per], dtype=float)
            res["scores"][k] = {"value": float(np.nanmean(v)) if np.isfinite(v).any() else float("nan")}
    elif mode == "context":
        ids = [i for i in ids if "cond" in run[i]]
        g = concat_marginals(marginals(*run[i]["cond"]) for i in ids)
        r = concat_marginals(marginals(*run[i]["real"]) for i in ids)
        res["scores"] = _summ(score(g, r, n_boot=n_boot))
    elif mode == "time_lagged":
        pairs = list(zip(ids[:-1], ids[1:]))
        g = concat_marginals(marginals(*run[a]["real"]) for a, _ in pairs)
        r = concat_marginals(marginals(*run[b]["real"]) for _, b in pairs)
        res["scores"] = _summ(score(g, r, n_boot=n_boot))
    elif mode == "divergence":
        res["buckets"] = []
        for k in range(buckets):
            def cut(x, k=k):
                n = len(x[0])
                lo, hi = k * n // buckets, (k + 1) * n // buckets
                return x[0][lo:hi], x[1][lo:hi]
            g = concat_marginals(marginals(*cut(run[i]["gen"])) for i in ids)
            r = concat_marginals(marginals(*cut(run[i]["real"])) for i in ids)
            res["buckets"].append(_summ(score(g, r, n_boot=0, distances=("wasserstein",))))
    else:
        raise ValueError(f"unknown mode {mode!r}")
    return res


def shard(windows: List[int], n_shards: int, k: int) -> List[int]:
    return [w for j, w in enumerate(sorted(windows)) if j % n_shards == k]


def merge(summaries: List[Dict]) -> Dict:
    """Window-weighted mean of per-shard summaries of the same mode."""
    tot = sum(s["n_windows"] for s in summaries)
    keys = summaries[0]["scores"].keys()
    return {"mode": summaries[0]["mode"], "n_windows": tot,
            "scores": {k: {"value": float(sum(s["scores"][k]["value"] * s["n_windows"] for s in summaries) / tot)}
                       for k in keys}}


def main(argv=None):
    p = argparse.ArgumentParser(description="score a generation run directory")
    p.add_argument("--save_dir", required=True)
    p.add_argument("--mode", default="uncond", choices=["uncond", "cond", "context", "time_lagged", "divergence"])
    p.add_argument("--n_boot", type=int, default=50)
    p.add_argument("--shards", type=int, default=1)
    p.add_argument("--shard", type=int, default=0)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    run = load_run(a.save_dir)
    wins = shard(list(run), a.shards, a.shard) if a.shards > 1 else None
    res = score_run(a.save_dir, a.mode, a.n_boot, windows=wins)
    txt = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(txt)
    else:
        print(txt)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
