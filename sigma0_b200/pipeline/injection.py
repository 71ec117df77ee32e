"""Verify a do(Q) injection from the generation CSVs alone (the J4 gate), with the
cross-arm diagnostics and a re-checkable report.

Between the generated book snapshots ``k-1`` and ``k`` (``data_gen`` orderbook
rows; row ``k`` is the book after message ``k``), the engine processed exactly
one message: the injected order.  For a passive limit order the L2 change must
be ``+qty`` at the injected price and nothing else inside the 10-level window
(the reference's ``lobpipeline/injection_verification.py`` J4; levels shifting
out of / into the window are tolerated).  Preconditions checked per window:
both books uncrossed and the injected price passive (below the best ask for a
bid, above the best bid for an ask).

``verify_arms`` adds, when reference runs are given (the reference's J0-J3 and J5, reported
but never gating, since they compare bytes across separate runs): J0 the same run twice is
byte-identical (P == P2), J1 injection off changes nothing (P == O), J2 the off and on arms
agree before the injected step, J3 the model's own message at the injected step is
unchanged and the provenance agrees through it, J5 the arms' books first differ exactly at
the injected step.  ``overall_pass`` reads J4 and its preconditions only.  ``check_report``
re-audits a written report's internal consistency without the data
(``python -m sigma0_b200.pipeline.injection --check REPORT``).
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import json
import os
import re
from typing import Dict, List, Optional

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


SCHEMA = "sigma0_b200.injection.v1"
_SUBDIRS = ("data_cond", "data_real", "data_gen")
_BLOCKS = ("j0_determinism", "j1_off_means_off", "j2_prefix", "j3_msg_row_k", "j4_book_injection",
           "j5_divergence")


def tree_digests(save_dir: str) -> Dict[str, str]:
    """SHA-256 of every file of a run's three data folders (one listing per folder)."""
    out = {}
    for sub in _SUBDIRS:
        d = os.path.join(save_dir, sub)
        if os.path.isdir(d):
            for f in sorted(os.listdir(d)):
                with open(os.path.join(d, f), "rb") as fh:
                    out[f"{sub}/{f}"] = hashlib.sha256(fh.read()).hexdigest()
    return out


def compare_trees(a: str, b: str, sub: Optional[str] = None) -> Dict:
    da, db = tree_digests(a), tree_digests(b)
    if sub:
        da = {k: v for k, v in da.items() if k.startswith(sub + "/")}
        db = {k: v for k, v in db.items() if k.startswith(sub + "/")}
    both = sorted(set(da) & set(db))
    mism = [k for k in both if da[k] != db[k]]
    only_a, only_b = sorted(set(da) - set(db)), sorted(set(db) - set(da))
    return {"pass": int(not mism and not only_a and not only_b and bool(both)), "n_files": len(both),
            "n_mismatch": len(mism), "mismatched_files": mism[:8], "only_a": only_a[:8], "only_b": only_b[:8]}


def _rows(path: str) -> List[str]:
    """Data lines of a CSV (the header row dropped)."""
    if not os.path.exists(path):
        return []
    with open(path) as f:
        lines = [ln.rstrip("\n") for ln in f if ln.strip()]
    return lines[1:]


def first_diff(a: List[str], b: List[str]) -> int:
    """First row where two row lists differ (-1: identical, lengths included)."""
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return -1 if len(a) == len(b) else min(len(a), len(b))


def _gen_windows(save_dir: str) -> Dict[int, Dict[str, str]]:
    out = {}
    for p in glob.glob(os.path.join(save_dir, "data_gen", "*_orderbook_real_id_*_gen_id_0.csv")):
        m = _GEN_OB.match(os.path.basename(p))
        if m:
            out[int(m["i"])] = {"orderbook": p, "message": p.replace("_orderbook_", "_message_"),
                                "provenance": p.replace("_orderbook_", "_provenance_")}
    return out


def verify_arms(dir_i: str, step: int, side: int, qty: int, offset_ticks: int, dir_o: Optional[str] = None,
                dir_p: Optional[str] = None, dir_p2: Optional[str] = None, tick: int = 100) -> Dict:
    """The full report: J4 on the injected arm (the gate) and the diagnostics J0-J3, J5 for
    whichever reference arms are given."""
    k = int(step)
    rep = {"schema": SCHEMA, "params": {"inject_step": k, "inject_side": side, "inject_qty": qty,
                                        "inject_price_offset_ticks": offset_ticks, "tick_size": tick},
           "inputs": {"dir_i": dir_i, "dir_o": dir_o, "dir_p": dir_p, "dir_p2": dir_p2}}
    skip = {"pass": 0, "skipped": 1}
    rep["j0_determinism"] = compare_trees(dir_p, dir_p2) if dir_p and dir_p2 else dict(skip)
    rep["j1_off_means_off"] = compare_trees(dir_p, dir_o) if dir_p and dir_o else dict(skip)
    j4 = verify_injection(dir_i, k, side, qty, offset_ticks, tick=tick)
    n_win = len(j4["windows"])
    n_pass = sum(int(w["ok"]) for w in j4["windows"])
    pre_fail = [w for w in j4["windows"] if not w["ok"] and any(
        t in w["reason"] for t in ("crossed", "passive", "indeterminate", "step 0"))]
    rep["j4_book_injection"] = {"pass": int(n_pass == n_win and n_win > 0), "n_windows": n_win,
                                "n_windows_pass": n_pass, "preconditions_pass": int(not pre_fail),
                                "per_window": j4["windows"]}
    if not dir_o:
        rep["j2_prefix"], rep["j3_msg_row_k"], rep["j5_divergence"] = dict(skip), dict(skip), dict(skip)
    else:
        wo, wi = _gen_windows(dir_o), _gen_windows(dir_i)
        if set(wo) != set(wi):
            err = {"pass": 0, "error": "the arms hold different windows"}
            rep["j2_prefix"], rep["j3_msg_row_k"], rep["j5_divergence"] = dict(err), dict(err), dict(err)
        else:
            j2 = j3 = prov = True
            fd_ob, fd_msg = [], []
            for w in sorted(wo):
                ob_o, ob_i = _rows(wo[w]["orderbook"]), _rows(wi[w]["orderbook"])
                ms_o, ms_i = _rows(wo[w]["message"]), _rows(wi[w]["message"])
                pv_o, pv_i = _rows(wo[w]["provenance"]), _rows(wi[w]["provenance"])
                j2 &= ob_o[:k] == ob_i[:k] and ms_o[:k] == ms_i[:k] and pv_o[:k] == pv_i[:k]
                j3 &= len(ms_o) > k and len(ms_i) > k and ms_o[k] == ms_i[k]
                prov &= pv_o[:k + 1] == pv_i[:k + 1]
                fd_ob.append(first_diff(ob_o, ob_i))
                fd_msg.append(first_diff(ms_o, ms_i))
            cond_eq = compare_trees(dir_o, dir_i, "data_cond")["pass"]
            real_eq = compare_trees(dir_o, dir_i, "data_real")["pass"]
            rep["j2_prefix"] = {"pass": int(j2 and cond_eq == 1 and real_eq == 1), "n_windows": len(wo),
                                "cond_tree_pass": cond_eq, "real_tree_pass": real_eq}
            rep["j3_msg_row_k"] = {"pass": int(j3), "n_windows": len(wo), "provenance_prefix_pass": int(prov)}
            rep["j5_divergence"] = {"pass": int(bool(fd_ob) and all(f == k for f in fd_ob)),
                                    "orderbook_first_divergence_min": min(fd_ob) if fd_ob else None,
                                    "orderbook_first_divergence_max": max(fd_ob) if fd_ob else None,
                                    "msg_first_divergence_per_window": fd_msg}
    rep["overall_pass"] = int(rep["j4_book_injection"]["pass"] == 1 and
                              rep["j4_book_injection"]["preconditions_pass"] == 1)
    return rep


def check_report(path: str) -> List[str]:
    """Internal consistency of a written report (no data needed): schema, every block present,
    the verdict equal to what its blocks imply, counts that add up, J5 at the injected step."""
    with open(path) as f:
        rep = json.load(f)
    if rep.get("schema") != SCHEMA:
        return [f"schema is {rep.get('schema')!r}, expected {SCHEMA!r}"]
    probs = [f"missing block: {b}" for b in _BLOCKS + ("params", "inputs", "overall_pass") if b not in rep]
    if probs:
        return probs
    j4 = rep["j4_book_injection"]
    want = int(j4.get("pass") == 1 and j4.get("preconditions_pass") == 1)
    if want != rep["overall_pass"]:
        probs.append(f"overall_pass={rep['overall_pass']} but the J4 block implies {want}")
    if j4.get("n_windows_pass") != sum(int(w.get("ok", 0)) for w in j4.get("per_window", [])):
        probs.append("J4 n_windows_pass disagrees with its per-window list")
    j5, k = rep["j5_divergence"], rep["params"].get("inject_step")
    if j5.get("pass") == 1 and (j5.get("orderbook_first_divergence_min") != k or
                                j5.get("orderbook_first_divergence_max") != k):
        probs.append("J5 passes but the books do not first differ at the injected step")
    return probs


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="verify a do(Q) injection run (J4 gate + diagnostics)")
    ap.add_argument("--dir_i", help="the injected run")
    ap.add_argument("--dir_o", default=None, help="the same run with injection off")
    ap.add_argument("--dir_p", default=None, help="a reference run (before the change)")
    ap.add_argument("--dir_p2", default=None, help="the reference run repeated")
    ap.add_argument("--step", type=int)
    ap.add_argument("--side", type=int)
    ap.add_argument("--qty", type=int)
    ap.add_argument("--offset_ticks", type=int)
    ap.add_argument("--tick", type=int, default=100)
    ap.add_argument("--out", default=None)
    ap.add_argument("--check", default=None, help="re-audit a written report instead")
    a = ap.parse_args(argv)
    if a.check:
        probs = check_report(a.check)
        print(json.dumps({"report": a.check, "problems": probs}))
        return int(bool(probs))
    rep = verify_arms(a.dir_i, a.step, a.side, a.qty, a.offset_ticks, a.dir_o, a.dir_p, a.dir_p2, a.tick)
    text = json.dumps(rep, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    print(json.dumps({k: rep[k].get("pass") for k in _BLOCKS} | {"overall_pass": rep["overall_pass"]}))
    return 0 if rep["overall_pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
