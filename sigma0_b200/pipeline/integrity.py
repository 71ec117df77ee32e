"""Content hashes and evidence records.

* ``tree_sha256`` -- one SHA-256 over a directory tree (sorted relative paths and
  file contents), the "merge record" of a vendored tree (reference
  ``lobpipeline/scorer/__init__.py:42-152``);
* ``record_evidence`` / ``check_evidence`` -- an evidence record is JSON holding
  the SHA-256 of named source files plus named assertions evaluated as data
  (``ci/record_evidence.py``, ``ci/check_evidence.py``): re-checking fails when a
  recorded file changed or an assertion no longer holds.  Assertions come in two forms:
  callables evaluated when the record is written, and declarative ones -- ``{"name",
  "metric": "dotted.path", "op": "<=", "value": ...}`` over the recorded ``metrics`` --
  that ``audit`` re-evaluates from the file itself, so a record whose numbers no longer
  satisfy its own conditions goes red without running anything;
* ``self_test`` plants each kind of defect (a drifted source, a failing, a malformed or an
  absent assertion, a record that asserts nothing) and requires every one to be caught:
  ``python -m sigma0_b200.pipeline.integrity --self-test``; ``audit FILE`` checks a record.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import operator
import os
import tempfile
from typing import Any, Callable, Dict, Iterable, List, Optional

OPS = {"==": operator.eq, "!=": operator.ne, "<": operator.lt, "<=": operator.le, ">": operator.gt,
       ">=": operator.ge}


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 20), b""):
            h.update(blk)
    return h.hexdigest()


def tree_sha256(root: str, ignore: Iterable[str] = ("__pycache__",)) -> str:
    h = hashlib.sha256()
    ign = set(ignore)
    for d, dirs, files in sorted(os.walk(root)):
        dirs[:] = sorted(x for x in dirs if x not in ign)
        for f in sorted(files):
            p = os.path.join(d, f)
            rel = os.path.relpath(p, root).replace(os.sep, "/")
            h.update(rel.encode() + b"\0")
            h.update(file_sha256(p).encode() + b"\n")
    return h.hexdigest()


def record_evidence(path: str, sources: Iterable[str], assertions: Dict[str, Callable[[], bool]],
                    meta: Dict = None, metrics: Optional[Dict] = None,
                    declared: Optional[List[Dict]] = None) -> Dict:
    rec = {"schema": "sigma0_b200.evidence.v1", "meta": meta or {},
           "sources": {s: file_sha256(s) for s in sources},
           "assertions": {k: bool(fn()) for k, fn in assertions.items()}}
    if metrics is not None or declared is not None:
        rec["metrics"] = metrics or {}
        rec["declared"] = list(declared or [])
    with open(path, "w") as f:
        json.dump(rec, f, indent=1, sort_keys=True)
    return rec


def check_evidence(path: str, assertions: Dict[str, Callable[[], bool]] = None) -> Dict[str, list]:
    with open(path) as f:
        rec = json.load(f)
    problems = {"changed": [], "missing": [], "failed": []}
    for s, h in rec["sources"].items():
        if not os.path.exists(s):
            problems["missing"].append(s)
        elif file_sha256(s) != h:
            problems["changed"].append(s)
    for k, ok in rec["assertions"].items():
        if not ok:
            problems["failed"].append(k)
    for k, fn in (assertions or {}).items():
        if not fn():
            problems["failed"].append(k)
    if "declared" in rec:
        problems["failed"] += declared_failures(rec)
    return problems


def _dig(obj: Any, dotted: str) -> Any:
    for k in dotted.split("."):
        obj = obj[int(k)] if isinstance(obj, list) else obj[k]
    return obj


def declared_failures(rec: Dict) -> List[str]:
    """Every declared assertion of ``rec`` that does not hold against its recorded metrics
    (a malformed or unknown-metric assertion, and a record that declares none, fail too)."""
    decl = rec.get("declared") or []
    if not decl:
        return ["the record declares no assertions, so it asserts nothing"]
    out = []
    for a in decl:
        name = a.get("name", "?")
        try:
            op = OPS[a["op"]]
            got = _dig(rec.get("metrics", {}), a["metric"])
            if not op(got, a["value"]):
                out.append(f"{name}: {a['metric']} = {got!r} is not {a['op']} {a['value']!r}")
        except KeyError as e:
            out.append(f"{name}: malformed or unknown ({e})")
        except (IndexError, TypeError, ValueError) as e:
            out.append(f"{name}: cannot evaluate ({e})")
    return out


def audit(path: str) -> Dict[str, list]:
    """``check_evidence`` of a record file, declarative assertions included."""
    return check_evidence(path)


def self_test() -> int:
    """Plant every kind of defect and require the audit to catch each one (0: all caught)."""
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "src.py")
        with open(src, "w") as f:
            f.write("x = 1\n")
        ok = [{"name": "x holds", "metric": "m.x", "op": "==", "value": 1}]
        cases = [
            ("a clean record passes", {"m": {"x": 1}}, ok, None, False),
            ("a drifted source is caught", {"m": {"x": 1}}, ok, "x = 2\n", True),
            ("a failing assertion is caught", {"m": {"x": 2}}, ok, None, True),
            ("a malformed assertion is caught", {"m": {"x": 1}}, [{"name": "bad", "metric": "m.x"}], None, True),
            ("an assertion on an absent metric is caught", {"m": {}}, ok, None, True),
            ("a record that asserts nothing is caught", {"m": {"x": 1}}, [], None, True),
        ]
        bad = []
        for title, metrics, declared, drift, must_fail in cases:
            with open(src, "w") as f:
                f.write("x = 1\n")
            path = os.path.join(d, "ev.json")
            record_evidence(path, [src], {}, metrics=metrics, declared=declared)
            if drift is not None:
                with open(src, "w") as f:
                    f.write(drift)
            p = audit(path)
            failed = bool(p["changed"] or p["missing"] or p["failed"])
            if failed != must_fail:
                bad.append(title)
        for t in bad:
            print(f"self-test: NOT as expected: {t}")
        if not bad:
            print("self-test passed: drift, failing, malformed, absent and missing assertions all go red")
        return 1 if bad else 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="evidence records: audit or self-test")
    ap.add_argument("files", nargs="*", help="evidence records to audit")
    ap.add_argument("--self-test", dest="self_test", action="store_true")
    a = ap.parse_args(argv)
    if a.self_test:
        return self_test()
    rc = 0
    for f in a.files:
        p = audit(f)
        bad = p["changed"] + p["missing"] + p["failed"]
        print(json.dumps({"file": f, **p}))
        rc |= int(bool(bad))
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
