"""Inspect and validate a checkpoint (native or Orbax layout) without restoring it into a
model: the reference's ``run/base_model/check_checkpoint.py`` with
``training/checkpoint_inspect.py:205-260``.

``python -m sigma0_b200.ckpt.inspect RUN_DIR [--step N] [--sample_arrays K] [--json]``

RUN_DIR is a checkpoint manager root (the newest step unless ``--step``) or a step directory.
The summary: the step and its paths, the layout, the model settings recorded in the
metadata (architecture, width, depth, sequence length, book input, optimizer), the number of
leaves and of parameters per top-level key (``params``, optimizer state, ...), and the
integrity check (file hashes of the native layout, every array present in the Orbax one).
``--sample_arrays K`` reads K arrays and reports their shape, dtype and a finiteness check.
"""
from __future__ import annotations

import argparse
import ast
import json
import os
from collections import Counter
from typing import Any, Dict, Optional

import numpy as np


def resolve_step(path: str, step: Optional[int] = None):
    """(manager root, step) of a manager root or a step directory."""
    path = os.path.abspath(path)
    base = os.path.basename(path)
    if base.isdigit() and os.path.isfile(os.path.join(path, "metadata", "metadata")):
        return os.path.dirname(path), int(base)
    from .checkpoint import CheckpointManager
    mgr = CheckpointManager.__new__(CheckpointManager)
    mgr.base = path
    steps = mgr.steps()
    if not steps:
        raise FileNotFoundError(f"no checkpoint steps under {path}")
    if step is not None and step not in steps:
        raise FileNotFoundError(f"step {step} not in {path} (have {steps})")
    return path, int(step if step is not None else steps[-1])


def _orbax_arrays(state_dir: str):
    with open(os.path.join(state_dir, "_METADATA")) as f:
        meta = json.load(f)
    for k in meta["tree_metadata"]:
        kp = tuple(ast.literal_eval(k))
        d = os.path.join(state_dir, ".".join(kp))
        shape = None
        for hdr in (".zarray", "zarr.json"):
            if os.path.exists(os.path.join(d, hdr)):
                with open(os.path.join(d, hdr)) as f:
                    shape = tuple(json.load(f)["shape"])
        yield kp, d, shape


def summarize(path: str, step: Optional[int] = None, sample_arrays: int = 0) -> Dict[str, Any]:
    from . import orbax as ox
    from .checkpoint import CheckpointManager
    root, step = resolve_step(path, step)
    step_dir = os.path.join(root, str(step))
    with open(os.path.join(step_dir, "metadata", "metadata")) as f:
        meta = json.load(f)
    cfg = meta.get("config", meta) if isinstance(meta, dict) else {}
    mgr = CheckpointManager.__new__(CheckpointManager)
    mgr.base = root
    out: Dict[str, Any] = {"manager_path": root, "step": step, "step_path": step_dir,
                           "layout": "orbax" if ox.is_orbax_step(step_dir) else "native",
                           "intact": bool(mgr.verify(step))}
    for k in ("architecture", "ssm_type", "model_type", "d_model", "n_layers", "n_messages", "msg_seq_len",
              "use_book_data", "opt_config", "token_mode"):
        if isinstance(cfg, dict) and k in cfg:
            out[k] = cfg[k]
    leaves, elements, samples = Counter(), Counter(), []
    if out["layout"] == "orbax":
        for kp, d, shape in _orbax_arrays(os.path.join(step_dir, "state")):
            leaves[kp[0]] += 1
            elements[kp[0]] += int(np.prod(shape)) if shape else 1
            if len(samples) < sample_arrays:
                a = ox.read_zarr(d) if os.path.exists(os.path.join(d, ".zarray")) else ox.read_zarr3(d)
                samples.append({"key": "/".join(kp), "shape": list(a.shape), "dtype": str(a.dtype),
                                "finite": bool(np.isfinite(a).all())})
    else:
        with open(os.path.join(step_dir, "state", "index.json")) as f:
            index = json.load(f)
        for leaf in index.get("leaves", []):
            top = leaf["path"].split("/")[0]
            leaves[top] += 1
            elements[top] += int(np.prod(leaf["shape"])) if leaf["shape"] else 1
        if sample_arrays:
            params = os.path.join(step_dir, "state", "params.f32")
            flat = np.fromfile(params, dtype="<f4") if os.path.exists(params) else None
            for leaf in index.get("leaves", [])[:sample_arrays]:
                n = int(np.prod(leaf["shape"])) if leaf["shape"] else 1
                entry = {"key": leaf["path"], "shape": leaf["shape"]}
                if flat is not None:
                    a = flat[leaf["offset"]:leaf["offset"] + n]
                    entry.update(dtype="float32", finite=bool(np.isfinite(a).all()))
                samples.append(entry)
    out["leaves"] = dict(leaves)
    out["elements"] = dict(elements)
    if samples:
        out["samples"] = samples
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="inspect and validate a checkpoint")
    ap.add_argument("checkpoint", help="checkpoint manager root or a step directory")
    ap.add_argument("--step", type=int, default=None)
    ap.add_argument("--sample_arrays", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    s = summarize(a.checkpoint, a.step, a.sample_arrays)
    if a.json:
        print(json.dumps(s, indent=1))
    else:
        for k, v in s.items():
            print(f"{k}: {v}")
    return 0 if s["intact"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
