"""Repository guards run as checks (the reference's ``ci/check_*.py``).

* ``non_english_lines`` -- source lines containing letters outside ASCII (the
  "english-only" guard: comments, identifiers and messages stay readable for
  every reviewer);
* ``forbidden_imports`` -- modules that must not be imported from product code
  (e.g. a legacy package, or a compatibility layer such as Triton);
* ``perplexity_decomposition_ok`` -- a message-perplexity report's ``full`` equals
  ``main + absolute_time + reference``.
"""
from __future__ import annotations

import ast
import os
import unicodedata
from typing import Dict, Iterable, List, Tuple


def _py_files(paths: Iterable[str]):
    for p in paths:
        if os.path.isdir(p):
            for d, _, fs in os.walk(p):
                for f in fs:
                    if f.endswith(".py"):
                        yield os.path.join(d, f)
        elif p.endswith(".py"):
            yield p


def non_english_lines(paths: Iterable[str]) -> List[Tuple[str, int, str]]:
    bad = []
    for f in _py_files(paths):
        for n, line in enumerate(open(f, encoding="utf-8"), 1):
            for ch in line:
                if ord(ch) > 127 and unicodedata.category(ch).startswith("L"):
                    bad.append((f, n, line.rstrip()))
                    break
    return bad


def forbidden_imports(paths: Iterable[str], forbidden: Iterable[str]) -> List[Tuple[str, int, str]]:
    forb = tuple(forbidden)
    bad = []
    for f in _py_files(paths):
        tree = ast.parse(open(f, encoding="utf-8").read(), f)
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom) and node.module and node.level == 0:
                names = [node.module]
            for nm in names:
                if any(nm == x or nm.startswith(x + ".") for x in forb):
                    bad.append((f, node.lineno, nm))
    return bad


def perplexity_decomposition_ok(report: Dict, tol: float = 1e-6) -> bool:
    roles = report["roles"]
    full = report["full"]["nats_per_message"]
    return abs(full - (roles["main"] + roles["absolute_time"] + roles["reference"])) <= tol * max(1.0, abs(full))
