"""Conditioning windows that end on a trade, for event-anchored evaluation: the reference's
``run/base_model/eval/pick_trade_anchors.py:82-245``.

    python -m sigma0_b200.eval.trade_anchors --data_dir DAYS --n_samples 1024 --out anchors.json
    python -m sigma0_b200.cli.infer ... --window_starts_file anchors.json

Windows on the dataset's fixed grid end on whatever message the grid gives (mostly
submissions and cancellations), so an event-anchored sample has to choose the window starts
itself.  Every execution (event type 4) at row ``r`` of a day gives the start
``r - n_cond_msgs + 1``, which puts the trade at the last conditioning position; a start is
usable when the whole ``n_cond_msgs + n_gen_msgs`` window and the book row after it fit in
the day.  The draw:

* takes at most one file per (ticker, trading day) -- the same day stored twice under
  different LOBSTER time ranges would count one execution twice -- unless
  ``--allow_duplicate_days``; the skipped files keep their positions, since ``file_idx`` is
  a position in the resolved file list (recorded in the output, which inference checks);
* balances the two trade directions (resting bid hit by a seller / resting ask lifted by a
  buyer) and makes up a shortfall on one side from the other;
* warns when fewer than five distinct days are drawn from: a day-block bootstrap over the
  anchors needs more.

Only columns 1 (event type) and 2 (direction: 1 = the resting order was on the bid) of the
memory-mapped message files are read.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
from collections import Counter
from typing import Dict, List, Sequence, Tuple

import numpy as np

TRADE = 4
SIDE_NAME = {1: "hit_bid_seller_initiated", 0: "lifted_ask_buyer_initiated"}


def one_file_per_day(msg_files: Sequence[str]) -> Tuple[set, Dict[str, int]]:
    """Indices of the first file of every (ticker, date) and the key -> index map."""
    first: Dict[str, int] = {}
    for i, f in enumerate(msg_files):
        base = os.path.basename(f)
        m = re.search(r"^([A-Za-z0-9.]+)_(\d{4}-\d{2}-\d{2})", base)
        key = f"{m.group(1)}_{m.group(2)}" if m else base
        first.setdefault(key, i)
    return set(first.values()), first


def candidate_anchors(msgs: np.ndarray, n_book_rows: int, n_cond: int, n_messages: int):
    """(window starts, trade directions, number of trades) of one day."""
    etype = np.asarray(msgs[:, 1])
    rows = np.flatnonzero(etype == TRADE)
    if rows.size == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64), 0
    last = min(msgs.shape[0], n_book_rows - 1)
    starts = rows - n_cond + 1
    fits = (starts >= 0) & (starts + n_messages <= last)
    return starts[fits].astype(np.int64), np.asarray(msgs[:, 2])[rows][fits].astype(np.int64), int(rows.size)


def stratified_take(rows: List[Tuple[int, int, int]], n: int, rng: np.random.Generator):
    """``n`` rows with the directions (third entry) as balanced as the pools allow."""
    pools: Dict[int, list] = {}
    for r in rows:
        pools.setdefault(r[2], []).append(r)
    sides = sorted(pools)
    per_side = {s: len(pools[s]) for s in sides}
    quota = n // max(1, len(sides))
    picked, rest = [], []
    for s in sides:
        order = rng.permutation(len(pools[s]))
        pool = [pools[s][i] for i in order]
        picked += pool[:quota]
        rest += pool[quota:]
    if len(picked) < n and rest:
        order = rng.permutation(len(rest))
        picked += [rest[i] for i in order[:n - len(picked)]]
    order = rng.permutation(len(picked))
    return [picked[i] for i in order][:n], per_side


def pick(msg_files: Sequence[str], book_files: Sequence[str], n_cond: int, n_gen: int, n_samples: int,
         seed: int = 42, allow_duplicate_days: bool = False, log=print) -> Dict:
    n_messages = n_cond + n_gen
    draw, first = one_file_per_day(msg_files)
    if allow_duplicate_days:
        draw = set(range(len(msg_files)))
    n_dup = len(msg_files) - len(first)
    if n_dup:
        log(f"duplicate days: {n_dup} extra file(s) " + ("included" if allow_duplicate_days else "skipped"))
    if len(draw) < 5:
        log(f"WARNING: only {len(draw)} trading day(s) to draw from; a day-block bootstrap needs more")
    rows, total, per_file = [], 0, []
    for i, (mf, bf) in enumerate(zip(msg_files, book_files)):
        if i not in draw:
            per_file.append([os.path.basename(mf), 0, 0])
            continue
        msgs = np.load(mf, mmap_mode="r")
        nb = np.load(bf, mmap_mode="r").shape[0]
        starts, dirs, nt = candidate_anchors(msgs, nb, n_cond, n_messages)
        total += nt
        per_file.append([os.path.basename(mf), nt, int(starts.size)])
        rows += [(i, int(s), int(d)) for s, d in zip(starts, dirs)]
    log(f"trades found: {total}; usable anchors: {len(rows)}")
    if not rows:
        raise ValueError("no usable trade anchors")
    picked, per_side = stratified_take(rows, n_samples, np.random.default_rng(seed))
    got = Counter(r[2] for r in picked)
    for s in sorted(per_side):
        log(f"direction={s} ({SIDE_NAME.get(s, '?')}): {got.get(s, 0)} selected of {per_side[s]}")
    if len(picked) < n_samples:
        log(f"NOTE: {n_samples - len(picked)} short of the {n_samples} requested")
    return {"n_cond_msgs": n_cond, "n_gen_msgs": n_gen, "n_messages": n_messages, "seed": seed,
            "distinct_days_drawn_from": len(first), "allow_duplicate_days": bool(allow_duplicate_days),
            "message_files": [os.path.abspath(f) for f in msg_files], "per_file": per_file,
            "windows": [[r[0], r[1]] for r in picked], "anchor_direction": [r[2] for r in picked],
            "direction_convention": "1 = resting bid (seller-initiated), 0 = resting ask (buyer-initiated)"}


def load_window_starts(path: str, msg_files: Sequence[str] = None) -> List[Tuple[int, int]]:
    """The ``(file_idx, seq_start)`` windows of an anchors file; with ``msg_files`` the file
    list it was drawn against must be the same (positions mean nothing otherwise)."""
    with open(path) as f:
        rec = json.load(f)
    if msg_files is not None and rec.get("message_files") is not None:
        have = [os.path.abspath(x) for x in msg_files]
        if have != rec["message_files"]:
            raise ValueError(f"{path} was drawn against another file list ({len(rec['message_files'])} files, "
                             f"resolved {len(have)})")
    return [(int(i), int(s)) for i, s in rec["windows"]]


def main(argv=None) -> int:
    from ..data.lobster import resolve_day_files
    ap = argparse.ArgumentParser(description="pick conditioning windows ending on a trade")
    ap.add_argument("--data_dir", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--n_cond_msgs", type=int, default=250)
    ap.add_argument("--n_gen_msgs", type=int, default=250)
    ap.add_argument("--n_samples", type=int, default=1024)
    ap.add_argument("--tickers", default=None)
    ap.add_argument("--date_range", default=None, help="START,END")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--allow_duplicate_days", action="store_true")
    a = ap.parse_args(argv)
    tickers = [t for t in a.tickers.split(",") if t] if a.tickers else None
    dates = tuple(a.date_range.split(",")) if a.date_range else None
    pairs = resolve_day_files(a.data_dir, tickers, dates)
    if not pairs:
        print(f"ERROR: no data files under {a.data_dir}", file=sys.stderr)
        return 1
    rec = pick([p[0] for p in pairs], [p[1] for p in pairs], a.n_cond_msgs, a.n_gen_msgs, a.n_samples, a.seed,
               a.allow_duplicate_days)
    rec["data_dir"] = os.path.abspath(a.data_dir)
    os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
    with open(a.out, "w") as f:
        json.dump(rec, f, indent=1)
    print(f"saved {a.out}: {len(rec['windows'])} windows")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
