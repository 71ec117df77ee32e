"""Flat ``key: value`` configuration files.

Same file format as the reference's launch configs (``src/base_model/config.py:14-50``,
``configs/train/*.yaml``) so those files can be read unchanged: one ``key: value``
per line, ``#`` comments, optional surrounding quotes, and a single-parent
``include: <path>`` (relative to the including file) whose values the child
overrides.  Keys prefixed ``env_`` are environment variables for the job.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Dict, Optional


def _unquote(v: str) -> str:
    if len(v) >= 2 and v[0] == v[-1] and v[0] in "'\"":
        return v[1:-1]
    return v


def read_flat_config(path, _chain: Optional[tuple] = None) -> Dict[str, str]:
    p = Path(path).resolve()
    chain = _chain or ()
    if p in chain:
        raise ValueError("config include cycle: " + " -> ".join(str(c) for c in chain + (p,)))
    if not p.exists():
        raise FileNotFoundError(f"config not found: {p}")
    out: Dict[str, str] = {}
    for n, raw in enumerate(p.read_text(encoding="utf-8").splitlines(), 1):
        line = raw.strip()
        if not line or line.startswith("#"):
            continue
        if ":" not in line:
            raise ValueError(f"{p}:{n}: expected 'key: value', got {raw!r}")
        k, v = line.split(":", 1)
        out[k.strip()] = _unquote(v.strip())
    inc = out.pop("include", None)
    if not inc:
        return out
    parent = Path(inc) if Path(inc).is_absolute() else p.parent / inc
    merged = read_flat_config(parent, chain + (p,))
    merged.update(out)
    return merged


def with_prefix(cfg: Dict[str, str], prefix: str) -> Dict[str, str]:
    """Entries whose key starts with ``prefix``, prefix removed (``env_`` -> environment)."""
    return {k[len(prefix):]: v for k, v in cfg.items() if k.startswith(prefix)}


def env_from_config(cfg: Dict[str, str], apply: bool = False) -> Dict[str, str]:
    env = with_prefix(cfg, "env_")
    if apply:
        os.environ.update(env)
    return env


def as_bool(v) -> bool:
    if isinstance(v, bool):
        return v
    return str(v).strip().lower() in ("1", "true", "yes", "on")


def coerce(v: str):
    """String -> bool/int/float/str, the way the launch scripts read env knobs."""
    s = str(v).strip()
    if s.lower() in ("true", "false"):
        return s.lower() == "true"
    for t in (int, float):
        try:
            return t(s)
        except ValueError:
            pass
    return s
