"""LOBSTER data: CSV import, day-file resolution, level selection, samplers.

* ``lobster_day_from_csv`` turns one LOBSTER day (message CSV ``Time, Type,
  OrderID, Size, Price, Direction`` and order-book CSV ``ask_p1, ask_v1,
  bid_p1, bid_v1, ...`` after each message) into the framework's day arrays:
  14-column message rows (relative price in ticks against the tick-floored mid
  before the message, inter-arrival time, and the referenced order's price,
  size and time for cancels / executions), per-message book rows
  ``[delta_mid, time_s, time_ns, L2...]`` describing the book *before* the
  message, engine rows and the opening L2 snapshot (the reference's
  ``jaxlobster`` loaders and ``preproc``, ``encoding_22tok.py:391``).
  Hidden executions, cross trades and trading halts (types 5, 6, 7) are
  dropped, as in ``df_msgs_to_jnp`` (``inference/generate.py:100``).
* ``save_day`` / ``LobWindowDataset.from_dir`` use ``<ticker>_<date>_message.npy``
  and ``..._book.npy``.
* ``resolve_day_files`` picks days by ticker and date range
  (``data/data_files.py:18``), from the data index ``build_index`` writes when one exists; ``select_levels`` cuts a wide (L500) book to L
  levels (``D5``); ``WindowSampler`` is the rank-interleaved, resumable,
  seeded sampler of ``data/dataloading.py:297``.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np

from ..encoding.tokenizer import NA_VAL

DROP_TYPES = (5, 6, 7)


@dataclass
class LobDay:
    msgs: np.ndarray          # (n, 14)
    books: np.ndarray         # (n, 3 + 4L) book before each message
    engine_msgs: np.ndarray   # (n, 8)
    l2_init: np.ndarray       # (4L,)


class MappedLobDay:
    """A day whose message and book arrays stay memory-mapped on disk (windows are read when
    a sample is drawn); the engine rows are built on first use only (training never needs
    them)."""

    def __init__(self, msgs: np.ndarray, books: np.ndarray):
        self.msgs, self.books = msgs, books
        self._engine = None
        self.l2_init = np.asarray(books[0, 3:], np.int64)

    @property
    def engine_msgs(self) -> np.ndarray:
        if self._engine is None:
            self._engine = raw_to_engine(np.asarray(self.msgs))
        return self._engine


def raw_to_engine(raw: np.ndarray) -> np.ndarray:
    """(n, 14) message rows -> (n, 8) engine rows [type, side, qty, price, oid, trader=0, sec, ns]
    (``msg_to_jnp``, ``inference/generate.py:118``)."""
    r = np.asarray(raw, dtype=np.int64)
    out = np.zeros((r.shape[0], 8), dtype=np.int64)
    out[:, 0] = r[:, 1]
    out[:, 1] = r[:, 2] * 2 - 1
    out[:, 2] = r[:, 5]
    out[:, 3] = r[:, 3]
    out[:, 4] = r[:, 0]
    out[:, 6] = r[:, 8]
    out[:, 7] = r[:, 9]
    return out


def _split_time(t: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """LOBSTER seconds-after-midnight (string or float) -> (s, ns) int64."""
    s_list, ns_list = [], []
    for v in t:
        txt = v if isinstance(v, str) else f"{float(v):.9f}"
        a, _, b = txt.partition(".")
        s_list.append(int(a))
        ns_list.append(int((b + "000000000")[:9]))
    return np.array(s_list, dtype=np.int64), np.array(ns_list, dtype=np.int64)


def _tick_mid(l2row: np.ndarray, tick: int, fallback: int) -> int:
    ap, bp = int(l2row[0]), int(l2row[2])
    if ap <= 0 or bp <= 0 or ap >= 9_999_999_999 or bp <= -9_999_999_999:
        return fallback
    return ((ap + bp) // 2 // tick) * tick


def lobster_day_from_arrays(time, etype, oid, size, price, direction, book: np.ndarray,
                            tick: int = 100, price_clip: int = 99_900) -> LobDay:
    """Columns of a LOBSTER message file + its (n, 4L) order-book rows (after each message)."""
    ts, tns = _split_time(np.asarray(time))
    etype = np.asarray(etype, dtype=np.int64)
    keep = ~np.isin(etype, DROP_TYPES)
    ts, tns, etype = ts[keep], tns[keep], etype[keep]
    oid = np.asarray(oid, dtype=np.int64)[keep]
    size = np.asarray(size, dtype=np.int64)[keep]
    price = np.asarray(price, dtype=np.int64)[keep]
    dirn = (np.asarray(direction, dtype=np.int64)[keep] + 1) // 2          # -1/1 -> 0/1
    book = np.asarray(book, dtype=np.int64)
    book_after = book[keep]
    n = len(etype)
    # book before message i = book after message i-1; the first uses the first row as the open
    l2_before = np.concatenate([book_after[:1], book_after[:-1]], 0)
    msgs = np.zeros((n, 14), dtype=np.int64)
    books = np.zeros((n, 3 + book.shape[1]), dtype=np.float64)
    t_ns = ts * 10**9 + tns
    dt = np.diff(t_ns, prepend=t_ns[:1])
    submitted: Dict[int, Tuple[int, int, int, int]] = {}
    prev_mid = _tick_mid(l2_before[0], tick, int(price[0]))
    for i in range(n):
        mid = _tick_mid(l2_before[i], tick, prev_mid)
        rel = int(np.clip(price[i] - mid, -price_clip, price_clip) // tick)
        ref = (NA_VAL, NA_VAL, NA_VAL, NA_VAL)
        if etype[i] == 1:
            submitted[int(oid[i])] = (rel, int(min(size[i], 9999)), int(ts[i]), int(tns[i]))
        elif int(oid[i]) in submitted:
            ref = submitted[int(oid[i])]
        msgs[i] = [oid[i], etype[i], dirn[i], price[i], rel, min(size[i], 9999), dt[i] // 10**9, dt[i] % 10**9,
                   ts[i], tns[i], *ref]
        books[i, 0] = (mid - prev_mid) / tick
        books[i, 1], books[i, 2] = ts[i], tns[i]
        books[i, 3:] = l2_before[i]
        prev_mid = mid
    return LobDay(msgs, books, raw_to_engine(msgs), l2_before[0].copy())


def lobster_day_from_csv(message_csv: str, book_csv: str, levels: Optional[int] = None, tick: int = 100) -> LobDay:
    import pandas as pd
    m = pd.read_csv(message_csv, header=None, dtype={0: str})
    b = pd.read_csv(book_csv, header=None).to_numpy()
    if levels is not None:
        b = select_levels(b, levels)
    return lobster_day_from_arrays(m[0].to_numpy(), m[1], m[2], m[3], m[4], m[5], b, tick)


def save_day(day: LobDay, directory: str, ticker: str, date: str) -> Tuple[str, str]:
    os.makedirs(directory, exist_ok=True)
    mp = os.path.join(directory, f"{ticker}_{date}_message.npy")
    bp = os.path.join(directory, f"{ticker}_{date}_book.npy")
    np.save(mp, day.msgs)
    np.save(bp, day.books)
    return mp, bp


def select_levels(wide: np.ndarray, levels: int) -> np.ndarray:
    """(n, 4*W) wide L2 rows -> the first ``levels`` levels (n, 4*levels)."""
    wide = np.asarray(wide)
    if wide.shape[-1] % 4:
        raise ValueError(f"wide-book width must be divisible by 4, found {wide.shape[-1]}")
    if 4 * levels > wide.shape[-1]:
        raise ValueError(f"asked for {levels} levels from a {wide.shape[-1] // 4}-level book")
    return wide[..., :4 * levels]


_DAY = re.compile(r"^(?P<ticker>[A-Za-z0-9.]+)_(?P<date>\d{4}-\d{2}-\d{2})_.*message.*\.npy(\.zst)?$")


INDEX_NAME = "index.json"


def _walk_day_files(root: str) -> List[str]:
    out = []
    for d, _, files in os.walk(root):
        for f in files:
            if _DAY.match(f):
                out.append(os.path.relpath(os.path.join(d, f), root))
    return sorted(out)


def build_index(root: str) -> Dict:
    """Write ``<root>/index.json``: every day file's relative path and array shape (read from
    the ``.npy`` header, no data loaded), so later runs find their days without walking the
    tree -- the reference's baked data index (``data/lobster_dataloader.py:55-114``), for
    filesystems where listing thousands of files is slow or forbidden."""
    files = {}
    for rel in _walk_day_files(root):
        for f in (rel, rel.replace("message", "book")):
            p = os.path.join(root, f)
            if os.path.exists(p):
                from .masks import load_npy
                files[f] = list(load_npy(p).shape)      # a header read for .npy, a decode for .npy.zst
    idx = {"schema": "sigma0_b200.data_index.v1", "shapes": files}
    tmp = os.path.join(root, INDEX_NAME + ".tmp")
    import json
    with open(tmp, "w") as fh:
        json.dump(idx, fh, indent=0, sort_keys=True)
    os.replace(tmp, os.path.join(root, INDEX_NAME))
    return idx


def load_index(root: str) -> Optional[Dict]:
    """The data index of ``root``: ``<root>/index.json``, else the file named by
    ``$DATA_INDEX_JSON``; None when there is none."""
    import json
    for p in (os.path.join(root, INDEX_NAME), os.environ.get("DATA_INDEX_JSON") or ""):
        if p and os.path.isfile(p):
            with open(p) as fh:
                return json.load(fh)
    return None


def resolve_day_files(root: str, tickers: Optional[Sequence[str]] = None,
                      date_range: Optional[Tuple[str, str]] = None) -> List[Tuple[str, str]]:
    """Paired ``(message.npy, book.npy)`` paths under ``root`` (recursive), filtered by
    ticker and inclusive ISO date range, ordered by (date, ticker).  With a data index the
    paths come from it and the tree is not walked."""
    idx = load_index(root)
    if idx is not None:
        out = []
        for rel in sorted(idx["shapes"]):
            f = os.path.basename(rel)
            m = _DAY.match(f)
            if not m or (tickers and m["ticker"] not in tickers):
                continue
            if date_range and not (date_range[0] <= m["date"] <= date_range[1]):
                continue
            brel = rel.replace("message", "book")
            if brel in idx["shapes"]:
                out.append((m["date"], m["ticker"], os.path.join(root, rel), os.path.join(root, brel)))
        out.sort()
        return [(a, b) for _, _, a, b in out]
    out = []
    for d, _, files in os.walk(root):
        for f in files:
            m = _DAY.match(f)
            if not m:
                continue
            if tickers and m["ticker"] not in tickers:
                continue
            if date_range and not (date_range[0] <= m["date"] <= date_range[1]):
                continue
            bf = f.replace("message", "book")
            if os.path.exists(os.path.join(d, bf)):
                out.append((m["date"], m["ticker"], os.path.join(d, f), os.path.join(d, bf)))
    out.sort()
    return [(a, b) for _, _, a, b in out]


class WindowSampler:
    """Rank-interleaved window indices: rank r of W takes windows r, r+W, ... of a
    seeded per-epoch permutation; ``start_step`` skips batches already consumed
    (resume), so a restarted job continues with the next unseen batch."""

    def __init__(self, n_windows: int, batch: int, world: int = 1, rank: int = 0, shuffle: bool = True,
                 seed: int = 0, start_step: int = 0, drop_last: bool = True):
        self.n, self.batch, self.world, self.rank = n_windows, batch, world, rank
        self.shuffle, self.seed, self.start_step, self.drop_last = shuffle, seed, start_step, drop_last

    def steps_per_epoch(self) -> int:
        per_rank = len(range(self.rank, self.n, self.world))
        return per_rank // self.batch if self.drop_last else -(-per_rank // self.batch)

    def epoch_indices(self, epoch: int) -> np.ndarray:
        order = np.random.default_rng(self.seed + epoch).permutation(self.n) if self.shuffle else np.arange(self.n)
        return order[self.rank::self.world]

    def __iter__(self) -> Iterator[List[int]]:
        spe = max(self.steps_per_epoch(), 1)
        step = self.start_step
        while True:
            ep, k = divmod(step, spe)
            idx = self.epoch_indices(ep)
            chunk = idx[k * self.batch:(k + 1) * self.batch]
            if len(chunk) == 0:
                return
            yield chunk.tolist()
            step += 1


def ticker_balanced_order(tickers: Sequence[str], seed: int = 0) -> np.ndarray:
    """Window order that alternates tickers round-robin (each ticker's windows in a
    seeded random order), so no ticker dominates a stretch of training."""
    rng = np.random.default_rng(seed)
    groups: Dict[str, List[int]] = {}
    for i, t in enumerate(tickers):
        groups.setdefault(t, []).append(i)
    lists = [list(rng.permutation(v)) for _, v in sorted(groups.items())]
    out = []
    while any(lists):
        for l in lists:
            if l:
                out.append(l.pop())
    return np.array(out, dtype=np.int64)


def make_snapshots(books: np.ndarray, times_ns: Sequence[int]) -> np.ndarray:
    """L2 snapshots at the given wall-clock times (ns since midnight): the book of the
    last event at or before each time (the wide-book snapshot builder of the
    reference's ``tools/data_build/make_snapshots.py``).  ``books`` rows are
    ``[dmid, time_s, time_ns, L2...]`` describing the book before each message, so the
    state *at* a message time is taken from the next row."""
    b = np.asarray(books)
    t = b[:, 1].astype(np.int64) * 1_000_000_000 + b[:, 2].astype(np.int64)
    idx = np.searchsorted(t, np.asarray(times_ns, dtype=np.int64), side="right")
    idx = np.clip(idx, 0, len(b) - 1)
    return b[idx, 3:]


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(description="LOBSTER day files: write the data index of a directory tree")
    ap.add_argument("--build_index", required=True, metavar="ROOT")
    a = ap.parse_args(argv)
    idx = build_index(a.build_index)
    print(f"{len(idx['shapes'])} files indexed in {os.path.join(a.build_index, INDEX_NAME)}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
