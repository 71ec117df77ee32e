"""Where a replayed window first disagrees with its recorded book, and what the message
there looks like -- a description of the divergence, not a repair (the reference's
"autopsy"; ``sim.autopsy`` here is the market maker's PnL split).

The reference's tool (``src/post_training/heuristic_learning/autopsy.py:77-179``) answers
one question per generated window: replaying the window's messages through the engine from
the conditioning book, at which step does our book first differ from the book the
generator (or the data, for the real arm) recorded, and which of a fixed set of
signatures does that step show.  Two choices carry it and are kept here:

* books are compared as (side, price) -> quantity maps, so one removed level reads as one
  change instead of a shift of every level below it;
* the deepest level is dropped before comparing, since a truncated L2 snapshot pulls new
  prices into view at its bottom edge when a level above disappears.  That edge effect
  cannot be removed completely, so one window's signature is evidence, not proof.

Signatures (several can hold at once, all are reported):

``RECORDED_NOT_APPLIED``  our replay moved, the recorded book did not
``APPLIED_NOT_RECORDED``  the recorded book moved, our replay did not
``DIFFERENT_PRICE``       both moved, at disjoint prices
``DIFFERENT_AMOUNT``      both moved at a shared price, by different amounts
``AGGRESSIVE_EXECUTION``  a type-4 execution: which resting orders it takes depends on
                          queue positions an L2 snapshot does not record
``MISS_SENTINEL``         the order id is the engine's lookup-miss sentinel
``OUT_OF_DEPTH``          the id names an initial order deeper than this replay created

Files are the generation runtime's layout (``cli/infer.py``): ``data_cond``,
``data_real`` and ``data_gen`` under the run directory, LOBSTER message CSVs (time as
``seconds.nanoseconds`` text, event type, order id, size, price, direction) and order-book
CSVs ``[ask_p, ask_v, bid_p, bid_v] x levels``; a header row is tolerated.

``python -m sigma0_b200.sim.divergence --run_dir RUN --stock SYN --date 2000-01-01 --index 0 3``
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Dict, List, Optional, Tuple

import numpy as np

from ..engine.book import NEGATIVE_RETURN_ID, EngineConfig
from .fidelity import replay_stream

EVENT_NAMES = {1: "NEW", 2: "PARTIAL_CANCEL", 3: "DELETE", 4: "EXECUTION"}
EMPTY_ASK = 2 ** 31 - 1


def run_paths(root: str, stock: str, date: str, index: int) -> Dict[str, str]:
    """The CSVs of generated window ``index`` of a generation run."""
    pre = f"{stock}_{date}"
    return {
        "cond_msg": os.path.join(root, "data_cond", f"{pre}_message_real_id_{index}.csv"),
        "cond_book": os.path.join(root, "data_cond", f"{pre}_orderbook_real_id_{index}.csv"),
        "real_msg": os.path.join(root, "data_real", f"{pre}_message_real_id_{index}.csv"),
        "real_book": os.path.join(root, "data_real", f"{pre}_orderbook_real_id_{index}.csv"),
        "gen_msg": os.path.join(root, "data_gen", f"{pre}_message_real_id_{index}_gen_id_0.csv"),
        "gen_book": os.path.join(root, "data_gen", f"{pre}_orderbook_real_id_{index}_gen_id_0.csv"),
    }


def _is_header(row: str) -> bool:
    """A header row: a field that is not a number (message files), or the column indices
    0, 1, 2, ... that pandas writes for an unnamed frame (book files)."""
    f = row.split(",")
    try:
        vals = [float(x) for x in f]
    except ValueError:
        return True
    return vals == [float(i) for i in range(len(vals))]


def _lines(path: str) -> List[str]:
    with open(path) as f:
        rows = [ln.strip() for ln in f if ln.strip()]
    return rows[1:] if rows and _is_header(rows[0]) else rows


def read_messages(path: str) -> np.ndarray:
    """A LOBSTER message CSV as (N, 8) engine rows ``(type, side, size, price, order_id,
    trader_id, time_s, time_ns)``.  The time is parsed as text so nanoseconds survive; the
    direction is taken as written (+1 / -1)."""
    rows = _lines(path)
    out = np.zeros((len(rows), 8), np.int64)
    for i, ln in enumerate(rows):
        t, typ, oid, size, price, direction = ln.split(",")[:6]
        sec, _, frac = t.partition(".")
        out[i] = (int(typ), int(direction), int(size), int(price), int(oid), 0, int(sec),
                  int((frac + "000000000")[:9]))
    return out


def read_books(path: str) -> np.ndarray:
    rows = _lines(path)
    b = np.array([[int(float(x)) for x in ln.split(",")] for ln in rows], np.int64).reshape(len(rows), -1)
    if b.shape[1] % 4:
        raise ValueError(f"{path}: {b.shape[1]} columns is not a multiple of 4")
    return b


def book_map(row: np.ndarray, drop_deepest: int = 1) -> Dict[Tuple[str, int], int]:
    """(side, price) -> quantity of an L2 row, the deepest ``drop_deepest`` levels left out;
    empty levels (the engine's sentinel prices) are skipped."""
    r = np.asarray(row, np.int64).reshape(-1, 4)
    out: Dict[Tuple[str, int], int] = {}
    for ap, av, bp, bv in r[:max(len(r) - drop_deepest, 0)]:
        if 0 < ap < EMPTY_ASK:
            out[("ask", int(ap))] = out.get(("ask", int(ap)), 0) + int(av)
        if bp > 0:
            out[("bid", int(bp))] = out.get(("bid", int(bp)), 0) + int(bv)
    return out


def book_delta(before: Dict, after: Dict) -> Dict[Tuple[str, int], int]:
    """Signed quantity change per (side, price); unchanged keys are omitted."""
    d = {k: after.get(k, 0) - before.get(k, 0) for k in set(before) | set(after)}
    return {k: v for k, v in d.items() if v}


def signatures(msg: np.ndarray, ref_d: Dict, our_d: Dict, n_levels: int,
               cfg: EngineConfig = EngineConfig()) -> List[str]:
    """The divergence signatures of one step (module docstring)."""
    out: List[str] = []
    typ, oid = int(msg[0]), int(msg[4])
    if our_d and not ref_d:
        out.append("RECORDED_NOT_APPLIED")
    if ref_d and not our_d:
        out.append("APPLIED_NOT_RECORDED")
    if ref_d and our_d:
        shared = set(ref_d) & set(our_d)
        if not shared:
            out.append("DIFFERENT_PRICE")
        elif set(ref_d) != set(our_d) or any(ref_d[k] != our_d[k] for k in shared):
            out.append("DIFFERENT_AMOUNT")
    if typ == 4:
        out.append("AGGRESSIVE_EXECUTION")
    lo_created = cfg.init_id - (2 * n_levels - 1)        # the init ids this replay creates
    if oid == NEGATIVE_RETURN_ID:
        out.append("MISS_SENTINEL")
    elif cfg.init_id - (2 * cfg.book_depth - 1) <= oid < lo_created:
        out.append("OUT_OF_DEPTH")
    return out or ["UNCLASSIFIED"]


def first_divergence(msgs: np.ndarray, ref_books: np.ndarray, init_l2: np.ndarray,
                     drop_deepest: int = 1, cfg: EngineConfig = EngineConfig()) -> Dict:
    """Replay ``msgs`` from ``init_l2`` and describe the first step whose book (as a price
    map) differs from ``ref_books`` (row i: the book after message i)."""
    init_l2 = np.asarray(init_l2, np.int64)
    n_levels = init_l2.shape[0] // 4
    ref_books = np.asarray(ref_books, np.int64)
    ours, report = replay_stream(msgs, init_l2, ref_books.shape[1] // 4, cfg)
    n = min(len(ours), len(ref_books))
    ref_maps = [book_map(ref_books[i], drop_deepest) for i in range(n)]
    our_maps = [book_map(ours[i], drop_deepest) for i in range(n)]
    k = next((i for i in range(n) if ref_maps[i] != our_maps[i]), -1)
    out = {"n_levels": n_levels, "n_steps": n, "first_step": k, "signatures": [],
           "replay_clean": report.clean}
    if k < 0:
        return out
    init_map = book_map(init_l2, drop_deepest)
    ref_d = book_delta(ref_maps[k - 1] if k else init_map, ref_maps[k])
    our_d = book_delta(our_maps[k - 1] if k else init_map, our_maps[k])
    m = np.asarray(msgs, np.int64)[k]
    key = lambda d: {f"{s}@{p}": q for (s, p), q in sorted(d.items())}
    out.update({
        "message": {"type": int(m[0]), "type_name": EVENT_NAMES.get(int(m[0]), "?"), "side": int(m[1]),
                    "qty": int(m[2]), "price": int(m[3]), "oid": int(m[4])},
        "ref_delta": key(ref_d), "our_delta": key(our_d),
        "disagreement": key(book_delta(our_maps[k], ref_maps[k])),
        "signatures": signatures(m, ref_d, our_d, n_levels, cfg),
    })
    return out


def autopsy_window(root: str, stock: str, date: str, index: int, arm: str = "gen") -> Optional[Dict]:
    """The first divergence of one window of a generation run (``arm``: ``gen`` replays the
    generated messages against the generator's books, ``real`` the data's continuation
    against the recorded books).  None when the window's files are missing."""
    p = run_paths(root, stock, date, index)
    mk, bk = ("real_msg", "real_book") if arm == "real" else ("gen_msg", "gen_book")
    if not all(os.path.isfile(p[x]) for x in (mk, bk, "cond_book")):
        return None
    cond = read_books(p["cond_book"])
    res = first_divergence(read_messages(p[mk]), read_books(p[bk]), cond[-1])
    res.update(window=f"{date} #{index}", arm=arm)
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--run_dir", required=True)
    ap.add_argument("--stock", default="SYN")
    ap.add_argument("--date", default="2000-01-01")
    ap.add_argument("--index", type=int, nargs="+", default=[0])
    ap.add_argument("--arm", choices=["gen", "real"], default="gen")
    a = ap.parse_args(argv)
    for i in a.index:
        res = autopsy_window(a.run_dir, a.stock, a.date, i, a.arm)
        print(json.dumps(res if res is not None else {"window": f"{a.date} #{i}", "missing": True}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
