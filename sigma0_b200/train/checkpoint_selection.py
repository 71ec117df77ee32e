"""Validation-only checkpoint selection for model comparisons.

The reference picks, from a run's checkpoints and their validation cross-entropy, the best
one and, for each target CE, the checkpoint closest to it ("iso-CE" comparison of models
of different sizes at equal validation loss), plus the step at which a run converged by
its 5,000-step / 1% rule (``src/base_model/training/checkpoint_selection.py:8-58``).
``evaluate_checkpoints`` produces the ``{step, validation_ce}`` rows from this package's
checkpoint directory.
"""
from __future__ import annotations

from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence


def select_checkpoints(results: Sequence[Dict[str, Any]], targets: Sequence[float],
                       tolerance: float) -> Dict[str, Any]:
    """``results``: rows ``{"step", "validation_ce"}``.  Returns the best-validation row and,
    per target (keyed by its 6-significant-digit string), the row closest to it (ties: the
    earlier step) with whether it is within ``tolerance`` and whether the run ever reached
    the target."""
    if not results:
        return {"best_validation": None, "iso_ce": {}}
    rows = sorted(results, key=lambda r: int(r["step"]))
    best = min(rows, key=lambda r: float(r["validation_ce"]))
    iso = {}
    for tgt in targets:
        near = min(rows, key=lambda r: abs(float(r["validation_ce"]) - tgt))
        delta = float(near["validation_ce"]) - tgt
        iso[format(tgt, ".6g")] = {
            "target": tgt, "step": int(near["step"]), "validation_ce": float(near["validation_ce"]),
            "delta": delta, "status": "matched" if abs(delta) <= tolerance else "outside_tolerance",
            "target_reached": float(best["validation_ce"]) <= tgt,
        }
    return {"best_validation": {"step": int(best["step"]), "validation_ce": float(best["validation_ce"])},
            "iso_ce": iso}


def convergence_step(results: Sequence[Dict[str, Any]], window: int = 5_000,
                     min_improvement: float = 0.01) -> Optional[int]:
    """The first step whose validation CE improved by less than ``min_improvement`` (relative)
    on the newest checkpoint at least ``window`` steps earlier; None if none has."""
    rows = sorted(results, key=lambda r: int(r["step"]))
    for cur in rows:
        earlier = [r for r in rows if int(r["step"]) <= int(cur["step"]) - window]
        if not earlier:
            continue
        prev = earlier[-1]
        gain = (float(prev["validation_ce"]) - float(cur["validation_ce"])) / float(prev["validation_ce"])
        if gain < min_improvement:
            return int(cur["step"])
    return None


def evaluate_checkpoints(ckpt_dir: str, make_trainer: Callable[[], Any], val_batches: Callable[[], Iterable],
                         steps: Optional[Sequence[int]] = None) -> List[Dict[str, Any]]:
    """Validation CE of every (or the given) checkpoint of ``ckpt_dir``: each one restored
    (parameters only) into a trainer from ``make_trainer`` and scored over ``val_batches()``."""
    from ..ckpt import CheckpointManager
    from .loop import evaluate
    tr = make_trainer()
    mgr = CheckpointManager(ckpt_dir, rank=tr.rank, world=tr.world)
    out = []
    for s in (steps if steps is not None else mgr.steps()):
        mgr.restore(tr, step=s, params_only=True)
        out.append({"step": int(s), "validation_ce": evaluate(tr, val_batches())})
    return out
