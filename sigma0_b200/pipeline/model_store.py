"""Model store: stable names pinned to checkpoint steps (reference ``lobpipeline/model_store.py:76-153``,
and the world-model pins of its market-making loop, ``post_training/heuristic_learning/
checkpoints.py:69-191``).

A JSON file maps a name to ``{"path", "step", "metadata_sha256", ...}`` plus free
fields (architecture, token mode, the pin's role and rationale).  ``resolve`` looks the name
up -- never a scan for the newest step -- and returns the entry after ``verify``: the step
directory exists, its metadata still hashes to the pinned value, the step passes the
checkpoint manager's integrity check (file hashes for the native layout, every array present
for the Orbax layout), and, only when asked (``require_latest``), no newer step exists.  A
name therefore cannot silently point at a different or damaged model.
"""
from __future__ import annotations

import json
import os
from typing import Dict

from .integrity import file_sha256


class ModelStoreError(RuntimeError):
    pass


def _meta_path(path: str, step: int) -> str:
    return os.path.join(path, str(step), "metadata", "metadata")


def pin(store: str, name: str, path: str, step: int, **info) -> Dict:
    mp = _meta_path(path, step)
    if not os.path.exists(mp):
        raise ModelStoreError(f"no checkpoint metadata at {mp}")
    pins = json.load(open(store)) if os.path.exists(store) else {}
    pins[name] = {"path": os.path.abspath(path), "step": int(step), "metadata_sha256": file_sha256(mp), **info}
    with open(store, "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
    return pins[name]


def verify(e: Dict, name: str = "", require_latest: bool = False) -> Dict:
    """``e`` itself when its pinned step is present, unchanged and intact; else ModelStoreError."""
    from ..ckpt.checkpoint import CheckpointManager
    mp = _meta_path(e["path"], e["step"])
    if not os.path.exists(mp) or file_sha256(mp) != e["metadata_sha256"]:
        raise ModelStoreError(f"pinned checkpoint for {name!r} changed or vanished ({mp})")
    mgr = CheckpointManager.__new__(CheckpointManager)    # read-only use: nothing is created
    mgr.base = e["path"]
    if not mgr.verify(int(e["step"])):
        raise ModelStoreError(f"pinned checkpoint for {name!r} fails its integrity check (step {e['step']})")
    if require_latest and mgr.latest_step() != int(e["step"]):
        raise ModelStoreError(f"pinned step {e['step']} of {name!r} is not the latest ({mgr.latest_step()})")
    return e


def resolve(store: str, name: str, require_latest: bool = False) -> Dict:
    pins = json.load(open(store))
    if name not in pins:
        raise ModelStoreError(f"unknown model {name!r}; pinned: {sorted(pins)}")
    return verify(pins[name], name, require_latest)
