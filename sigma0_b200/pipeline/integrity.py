"""Content hashes and evidence records.

* ``tree_sha256`` -- one SHA-256 over a directory tree (sorted relative paths and
  file contents), the "merge record" of a vendored tree (reference
  ``lobpipeline/scorer/__init__.py:42-152``);
* ``record_evidence`` / ``check_evidence`` -- an evidence record is JSON holding
  the SHA-256 of named source files plus named assertions evaluated as data
  (``ci/record_evidence.py``, ``ci/check_evidence.py``): re-checking fails when a
  recorded file changed or an assertion no longer holds.
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Callable, Dict, Iterable


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
                    meta: Dict = None) -> Dict:
    rec = {"schema": "sigma0_b200.evidence.v1", "meta": meta or {},
           "sources": {s: file_sha256(s) for s in sources},
           "assertions": {k: bool(fn()) for k, fn in assertions.items()}}
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
    return problems
