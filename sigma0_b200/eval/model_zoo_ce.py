"""Validation CE of every checkpoint of a run on one fixed held-out sample, with the iso-CE
checkpoint selection: the reference's ``run/base_model/evaluate_model_zoo_ce.py:73-270``.

    python -m sigma0_b200.eval.model_zoo_ce --checkpoint_root RUN/ck --data_dir DAYS \\
        --tickers GOOG --date_range 2025-12-01,2025-12-31 --output zoo_ce.json

* the steps are the complete ones under the root (a ``state/`` directory and
  ``metadata/metadata``), all or ``--steps 1000,2000``; a requested step that is missing or
  incomplete is an error;
* the model comes from the first step's recorded config; every other step must record the
  same architecture, width, depth, token mode and seed (config drift is an error), and
  ``--expected_architecture`` / ``--expected_seed`` are checked against it;
* the held-out sample (``--max_batches`` batches of ``--batch_size`` windows, seeded) is
  drawn ONCE and reused for every checkpoint, so the CEs are comparable;
* after each step the JSON record is rewritten atomically: per-step validation CE and
  next-token accuracy, the best-validation and iso-CE selection at ``--targets``
  (``train/checkpoint_selection.py``) and the convergence step.
"""
from __future__ import annotations

import argparse
import json
import os
from types import SimpleNamespace
from typing import Any, Dict, List, Optional, Sequence

import numpy as np
import torch

DRIFT_KEYS = ("architecture", "d_model", "n_layers", "token_mode", "seed")


def complete_steps(root: str) -> List[int]:
    steps = sorted(int(n) for n in os.listdir(root) if n.isdigit()
                   and os.path.isdir(os.path.join(root, n, "state"))
                   and os.path.isfile(os.path.join(root, n, "metadata", "metadata")))
    if not steps:
        raise ValueError(f"no complete checkpoint steps under {root}")
    return steps


def step_config(root: str, step: int) -> Dict[str, Any]:
    with open(os.path.join(root, str(step), "metadata", "metadata")) as f:
        meta = json.load(f)
    if not isinstance(meta, dict) or "config" not in meta:
        raise ValueError(f"checkpoint step {step} records no config")
    cfg = dict(meta["config"])
    if "seed" not in cfg and "jax_seed" in cfg:
        cfg["seed"] = cfg["jax_seed"]
    return cfg


def check_configs(root: str, steps: Sequence[int], expected_architecture: Optional[str] = None,
                  expected_seed: Optional[int] = None) -> Dict[str, Any]:
    cfg = step_config(root, steps[0])
    if expected_architecture is not None and cfg.get("architecture") != expected_architecture:
        raise ValueError(f"checkpoint architecture mismatch: expected {expected_architecture!r}, "
                         f"got {cfg.get('architecture')!r}")
    if expected_seed is not None and (cfg.get("seed") is None or int(cfg["seed"]) != expected_seed):
        raise ValueError(f"checkpoint seed mismatch: expected {expected_seed}, got {cfg.get('seed')!r}")
    for s in steps[1:]:
        other = step_config(root, s)
        for k in DRIFT_KEYS:
            if other.get(k) != cfg.get(k):
                raise ValueError(f"checkpoint config drift at step {s}: {k}")
    return cfg


def model_args_from_config(cfg: Dict[str, Any], batch_size: int):
    from ..models.presets import _DEFAULTS
    d = dict(_DEFAULTS)
    d.update(cfg)
    d["micro_bsz"] = batch_size
    return SimpleNamespace(**d)


def fixed_sample(days, args, batch_size: int, max_batches: int, seed: int = 42):
    """``max_batches`` batches drawn once without replacement (seeded), kept in host memory."""
    from ..data import LobWindowDataset, collate
    ds = LobWindowDataset.from_days(days, args.n_messages, token_mode=args.token_mode)
    need = batch_size * max_batches
    if len(ds) < need:
        raise ValueError(f"the held-out data has {len(ds)} windows, fewer than the fixed sample of {need}")
    order = np.random.default_rng(seed).permutation(len(ds))[:need]
    return [collate([ds[int(i)] for i in order[b * batch_size:(b + 1) * batch_size]]) for b in range(max_batches)]


def accuracy(model, batches) -> float:
    dev = next(model.parameters()).device
    hit = tot = 0
    with torch.no_grad():
        for tokens, labels, book in batches:
            logp = model(tokens.to(dev), book.to(dev) if book is not None else None)
            lab = labels.to(dev)
            ok = lab >= 0
            hit += int(((logp.argmax(-1) == lab) & ok).sum())
            tot += int(ok.sum())
    return hit / max(tot, 1)


def _write_json(path: str, payload: Dict[str, Any]) -> None:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(payload, f, indent=2, sort_keys=True)
        f.write("\n")
    os.replace(tmp, path)


def main(argv=None) -> int:
    from ..ckpt import CheckpointManager
    from ..cli.common import load_days
    from ..train.checkpoint_selection import convergence_step, select_checkpoints
    from ..train.loop import evaluate
    from ..train.trainer import Trainer
    p = argparse.ArgumentParser(description="validation CE of every checkpoint on a fixed held-out sample")
    p.add_argument("--checkpoint_root", required=True)
    p.add_argument("--expected_architecture", default=None)
    p.add_argument("--expected_seed", type=int, default=None)
    p.add_argument("--data_dir", default=None)
    p.add_argument("--synthetic", type=int, default=0, help="seeded synthetic days instead of --data_dir")
    p.add_argument("--tickers", default=None)
    p.add_argument("--date_range", default=None, help="START,END")
    p.add_argument("--batch_size", type=int, default=8)
    p.add_argument("--max_batches", type=int, default=8)
    p.add_argument("--targets", default="0.70,0.65,0.60")
    p.add_argument("--target_tolerance", type=float, default=0.01)
    p.add_argument("--steps", default="all", help="all or comma-separated checkpoint steps")
    p.add_argument("--output", required=True)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = p.parse_args(argv)
    if a.batch_size < 1 or a.max_batches < 1:
        p.error("batch_size and max_batches must be positive")
    dates = None
    if a.date_range:
        dates = tuple(x.strip() for x in a.date_range.split(","))
        if len(dates) != 2:
            p.error("date_range must be START,END")
    tickers = [t.strip() for t in a.tickers.split(",") if t.strip()] if a.tickers else None
    targets = [float(x) for x in a.targets.split(",") if x.strip()]
    have = complete_steps(a.checkpoint_root)
    if a.steps == "all":
        steps = have
    else:
        want = sorted({int(x) for x in a.steps.split(",") if x.strip()})
        missing = sorted(set(want) - set(have))
        if missing:
            raise ValueError(f"requested missing or incomplete checkpoint steps: {missing}")
        steps = want
    cfg = check_configs(a.checkpoint_root, steps, a.expected_architecture, a.expected_seed)
    args = model_args_from_config(cfg, a.batch_size)
    days = load_days(a.data_dir, a.synthetic or 2, args.n_messages * 4 + 1, 0, tickers=tickers, date_range=dates)
    batches = fixed_sample(days, args, a.batch_size, a.max_batches)
    tr = Trainer(args, device=torch.device(a.device))
    mgr = CheckpointManager(a.checkpoint_root)
    payload: Dict[str, Any] = {
        "schema_version": 1, "checkpoint_root": os.path.abspath(a.checkpoint_root),
        "architecture": cfg.get("architecture"), "seed": cfg.get("seed"), "token_mode": cfg.get("token_mode"),
        "validation": {"tickers": tickers, "date_range": list(dates) if dates else None,
                       "batch_size": a.batch_size, "max_batches": a.max_batches, "sampling_seed": 42,
                       "sampling": "fixed sample without replacement, drawn once",
                       "sequences": a.batch_size * a.max_batches,
                       "token_values": int(sum(b[0].numel() for b in batches))},
        "targets": targets, "target_tolerance": a.target_tolerance, "results": [],
        "selection": {"best_validation": None, "iso_ce": {}}, "convergence_step": None}
    for s in steps:
        mgr.restore(tr, step=s, params_only=True)
        tr.model.eval()
        row = {"step": int(s), "validation_ce": evaluate(tr, batches), "validation_accuracy": accuracy(tr.model, batches)}
        payload["results"].append(row)
        payload["selection"] = select_checkpoints(payload["results"], targets, a.target_tolerance)
        payload["convergence_step"] = convergence_step(payload["results"])
        _write_json(a.output, payload)
        print(f"[ce-eval] step={s} validation_ce={row['validation_ce']:.8f} "
              f"accuracy={row['validation_accuracy']:.8f}", flush=True)
    print(f"[ce-eval] wrote {a.output}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
