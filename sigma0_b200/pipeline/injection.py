"""Verify a do(Q) injection from the generation CSVs alone (the J4 gate).

Between the generated book snapshots ``k-1`` and ``k`` (``data_gen`` orderbook
rows; row ``k`` is the book after message ``k``), the engine processed exactly
one message: the injected order.  For a passive limit order the L2 change must
be ``+qty`` at the injected price and nothing else inside the 10-level window
(the reference's ``lobpipeline/injection_verification.py`` J4; levels shifting
out of / into the window are tolerated).  Preconditions checked per window:
both books uncrossed and the injected price passive (below the best ask for a
bid, above the best bid for an ask).
"""
from __future__ import annotations

import glob
import os
import re
from typing import Dict, List

import numpy as np

EMPTY_ASK_P = 2_147_483_647
EMPTY_BID_P = -2_147_483_647
_GEN_OB = re.compile(r"^(?P<stock>.+)_(?P<date>\d{4}-\d{2}-\d{2})_orderbook_real_id_(?P<i>\d+)_gen_id_0\.csv$")


def _levels(row: np.ndarray, side: int) -> Dict[int, int]:
    """{price: volume} of one side (0 ask, 1 bid) of an L2 row."""
    p = row[2 * side::4]
    v = row[2 * side + 1::4]
    return {int(a): int(b) for a, b in zip(p, v) if a not in (EMPTY_ASK_P, EMPTY_BID_P)}


def check_window(books: np.ndarray, step: int, side: int, qty: int, price: int) -> Dict:
    before, after = books[step - 1] if step > 0 else None, books[step]
    if before is None:
        return {"ok": False, "reason": "injection at step 0 has no generated book before it"}
    res = {"ok": True, "reason": ""}
    for tag, b in (("before", before), ("after", after)):
        if b[0] != EMPTY_ASK_P and b[2] != EMPTY_BID_P and b[0] <= b[2]:
            return {"ok": False, "reason": f"crossed book {tag}"}
    if (side == 1 and price >= before[0]) or (side == 0 and price <= before[2]):
        return {"ok": False, "reason": "injected price is not passive"}
    sd = 1 if side == 1 else 0
    lb, la = _levels(before, sd), _levels(after, sd)
    delta = {p: la.get(p, 0) - lb.get(p, 0) for p in set(lb) | set(la)}
    # levels that appear or vanish at the edge of the 10-level window are not compared
    changed = {p: d for p, d in delta.items() if d != 0}
    if changed.get(price) != qty:
        return {"ok": False, "reason": f"expected +{qty} at {price}, saw {changed.get(price, 0)}"}
    others = {p: d for p, d in changed.items() if p != price and p in lb and p in la}
    if others:
        return {"ok": False, "reason": f"other levels changed: {others}"}
    other_side = _levels(before, 1 - sd), _levels(after, 1 - sd)
    common = set(other_side[0]) & set(other_side[1])
    if any(other_side[0][p] != other_side[1][p] for p in common):
        return {"ok": False, "reason": "the opposite side changed"}
    return res


def verify_injection(save_dir: str, step: int, side: int, qty: int, offset_ticks: int, mids: Dict[int, int] = None,
                     tick: int = 100) -> Dict:
    """J4 over every generated window of ``save_dir``; ``mids[i]`` is the tick-floored mid
    before the injected step of window ``i`` (the price is ``mid + offset * tick``).
    Without ``mids`` the generator's own mid sidecar (``mid_after`` of the provenance
    CSV, step ``k - 1``) is used, else the mid of book row ``k - 1`` (which must then
    have both sides: an indeterminate mid fails the window)."""
    import pandas as pd
    out: List[Dict] = []
    for p in sorted(glob.glob(os.path.join(save_dir, "data_gen", "*_orderbook_real_id_*_gen_id_0.csv"))):
        m = _GEN_OB.match(os.path.basename(p))
        i = int(m["i"])
        books = pd.read_csv(p).to_numpy().astype(np.int64)
        side_car = p.replace("_orderbook_", "_provenance_")
        if mids and i in mids:
            mid = mids[i]
        elif os.path.exists(side_car) and "mid_after" in pd.read_csv(side_car).columns:
            mid = int(pd.read_csv(side_car)["mid_after"].iloc[step - 1])
        else:
            b = books[step - 1]
            if b[0] == EMPTY_ASK_P or b[2] == EMPTY_BID_P:
                out.append({"ok": False, "reason": "indeterminate mid (one-sided book)", "window": i})
                continue
            mid = (int(b[0]) + int(b[2])) // 2 // tick * tick
        r = check_window(books, step, side, qty, mid + offset_ticks * tick)
        r["window"] = i
        out.append(r)
    return {"J4": all(r["ok"] for r in out) and bool(out), "windows": out}
