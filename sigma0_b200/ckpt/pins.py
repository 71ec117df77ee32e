"""Pinned checkpoints: a named (directory, step) fixed by the SHA-256 of its metadata, so
a closed-loop experiment keeps using exactly the world model it was set up with.

The reference pins the two world models of its market-making loop -- one chosen for the
background order flow (best distributional fit), one for the price signal (best direction
accuracy), deliberately different steps of different runs and neither the latest
(``src/post_training/heuristic_learning/checkpoints.py:69-191``).  The contract kept here:
a pin is looked up by name, never by scanning for the newest step; ``verify`` fails loudly
(``CheckpointDrift``) when the step is missing, incomplete or its metadata changed, and
checks freshness only when asked (``require_latest``).  The pins live in a JSON registry
file instead of the reference's hard-coded cluster paths; a step's completeness is the
checkpoint manager's own integrity check (file hashes for the native layout, every array
present for the Orbax layout).
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import asdict, dataclass
from typing import Dict, Optional


class CheckpointDrift(RuntimeError):
    """A pinned checkpoint is missing, incomplete or no longer the one that was pinned."""


@dataclass(frozen=True)
class CheckpointPin:
    name: str
    ckpt_dir: str
    step: int
    metadata_sha256: str
    role: str = ""
    rationale: str = ""

    @property
    def step_dir(self) -> str:
        return os.path.join(self.ckpt_dir, str(self.step))


def metadata_sha256(ckpt_dir: str, step: int) -> str:
    """SHA-256 of ``<ckpt_dir>/<step>/metadata/metadata``."""
    with open(os.path.join(ckpt_dir, str(step), "metadata", "metadata"), "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def pin(name: str, ckpt_dir: str, step: int, role: str = "", rationale: str = "") -> CheckpointPin:
    """Pin an existing, complete step of ``ckpt_dir`` under ``name``."""
    p = CheckpointPin(name, os.path.abspath(ckpt_dir), int(step), metadata_sha256(ckpt_dir, step), role, rationale)
    return verify(p)


def verify(p: CheckpointPin, require_latest: bool = False) -> CheckpointPin:
    """``p`` itself when its step is present, complete and unchanged; else CheckpointDrift.
    ``require_latest`` also demands that no newer step exists in the directory (one listing)."""
    from .checkpoint import CheckpointManager
    if not os.path.isdir(p.step_dir):
        raise CheckpointDrift(f"{p.name}: step directory absent: {p.step_dir}")
    if not os.path.isfile(os.path.join(p.step_dir, "metadata", "metadata")):
        raise CheckpointDrift(f"{p.name}: incomplete checkpoint (no metadata/metadata) in {p.step_dir}")
    got = metadata_sha256(p.ckpt_dir, p.step)
    if got != p.metadata_sha256:
        raise CheckpointDrift(f"{p.name}: metadata changed since it was pinned "
                              f"(pinned {p.metadata_sha256[:12]}..., now {got[:12]}...)")
    mgr = CheckpointManager.__new__(CheckpointManager)    # read-only use: no directory creation
    mgr.base = p.ckpt_dir
    if not mgr.verify(p.step):
        raise CheckpointDrift(f"{p.name}: step {p.step} fails its integrity check")
    if require_latest:
        latest = mgr.latest_step()
        if latest != p.step:
            raise CheckpointDrift(f"{p.name}: pinned step {p.step} is not the latest ({latest})")
    return p


class PinRegistry:
    """Named pins kept in one JSON file (``{name: pin fields}``)."""

    def __init__(self, path: str):
        self.path = path
        self.pins: Dict[str, CheckpointPin] = {}
        if os.path.isfile(path):
            with open(path) as f:
                self.pins = {k: CheckpointPin(**v) for k, v in json.load(f).items()}

    def add(self, p: CheckpointPin) -> None:
        self.pins[p.name] = p
        tmp = self.path + ".tmp"
        with open(tmp, "w") as f:
            json.dump({k: asdict(v) for k, v in sorted(self.pins.items())}, f, indent=1)
        os.replace(tmp, self.path)

    def resolve(self, name: str, verify_now: bool = True, require_latest: bool = False) -> CheckpointPin:
        """The pin called ``name`` (a lookup, never a scan for the newest step)."""
        if name not in self.pins:
            raise KeyError(f"unknown checkpoint pin {name!r}; known pins: {', '.join(sorted(self.pins))}")
        p = self.pins[name]
        return verify(p, require_latest) if verify_now else p


def resolve(registry_path: str, name: str, require_latest: bool = False) -> CheckpointPin:
    return PinRegistry(registry_path).resolve(name, True, require_latest)


def describe(p: CheckpointPin) -> Dict[str, Optional[str]]:
    return {**asdict(p), "step_dir": p.step_dir}
