"""Model store: stable names pinned to checkpoint steps (reference ``lobpipeline/model_store.py:76-153``).

A JSON file maps a name to ``{"path", "step", "architecture", "token_mode",
"metadata_sha256"}``; ``resolve`` returns the entry after checking that the
checkpoint's metadata still hashes to the pinned value, so a name cannot
silently point at a different model.
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


def resolve(store: str, name: str) -> Dict:
    pins = json.load(open(store))
    if name not in pins:
        raise ModelStoreError(f"unknown model {name!r}; pinned: {sorted(pins)}")
    e = pins[name]
    mp = _meta_path(e["path"], e["step"])
    if not os.path.exists(mp) or file_sha256(mp) != e["metadata_sha256"]:
        raise ModelStoreError(f"pinned checkpoint for {name!r} changed or vanished ({mp})")
    return e
