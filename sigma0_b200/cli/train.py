"""Training runtime: one process per GPU (torchrun), optional flat config file.

    torchrun --nproc-per-node 8 -m sigma0_b200.cli train --preset 350m --data_dir <days> \
        --ckpt_dir <dir> --steps 10000 --dp_impl fused

``--config`` reads a flat ``key: value`` file (``include:`` supported); its
``env_*`` keys are exported to the environment and its plain keys override
argument defaults (the reference's launch configs work unchanged for the keys
both sides know).  Mirrors ``run/base_model/runtime/train.py:47-330``: model
and optimizer flags, data selection, checkpointing/resume, watchdog, and the
distributed options (replicated / sharded / fused gradient sync, bf16 wire,
gradient accumulation, and ``--context_parallel``, which splits every sequence over the
ranks instead of the batch).
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np
import torch

from .common import add_model_args, dist_env, load_days, model_args


def parse(argv=None):
    p = argparse.ArgumentParser(description="sigma0-b200 training runtime")
    p.add_argument("--config", default=None)
    add_model_args(p)
    p.add_argument("--data_dir", default=None)
    p.add_argument("--tickers", default=None, help="comma-separated")
    p.add_argument("--train_date_range", default=None, help="YYYY-MM-DD,YYYY-MM-DD")
    p.add_argument("--synthetic", type=int, default=8, help="synthetic days when no --data_dir")
    p.add_argument("--n_messages", type=int, default=None)
    p.add_argument("--micro_bsz", type=int, default=None)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--lr", type=float, default=None, help="ssm_lr_base")
    p.add_argument("--lr_factor", type=float, default=None)
    p.add_argument("--weight_decay", type=float, default=None)
    p.add_argument("--warmup_end", type=float, default=None)
    p.add_argument("--opt_config", default=None)
    p.add_argument("--ignore_times", action="store_true")
    p.add_argument("--ckpt_dir", default=None)
    p.add_argument("--save_every", type=int, default=0)
    p.add_argument("--ckpt_format", choices=["native", "orbax"], default="native",
                   help="native flat buffers, or the Orbax StandardSave layout (zarr arrays by Flax path)")
    p.add_argument("--no_resume", action="store_true")
    p.add_argument("--log_every", type=int, default=100)
    p.add_argument("--watchdog_timeout", type=float, default=900.0)
    p.add_argument("--time_limit_s", type=float, default=None)
    p.add_argument("--dp_impl", choices=["nccl", "fused"], default="nccl")
    p.add_argument("--sharded", action="store_true")
    p.add_argument("--grad_wire_dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--accum_steps", type=int, default=1)
    p.add_argument("--tp", type=int, default=1,
                   help="tensor-parallel size: heads split over groups of --tp consecutive ranks, batch over the rest")
    p.add_argument("--context_parallel", action="store_true",
                   help="split every sequence over the ranks (message-aligned segments) instead of the batch")
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    if a.config:
        from ..utils.config import coerce, env_from_config, read_flat_config
        cfg = read_flat_config(a.config)
        env_from_config(cfg, apply=True)
        explicit = {x.split("=")[0].lstrip("-") for x in (argv if argv is not None else sys.argv[1:])
                    if x.startswith("--")}
        for k, v in cfg.items():
            if hasattr(a, k) and k not in explicit and not k.startswith("env_"):
                setattr(a, k, coerce(v))
    return a


def main(argv=None):
    from ..data import LobWindowDataset, collate
    from ..data.lobster import WindowSampler
    from ..train.loop import LoopConfig, fit
    from ..train.trainer import Trainer
    a = parse(argv)
    rank, world, local = dist_env()
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
            dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    extra = {k: v for k, v in (("n_messages", a.n_messages), ("micro_bsz", a.micro_bsz), ("ssm_lr_base", a.lr),
                               ("lr_factor", a.lr_factor), ("weight_decay", a.weight_decay),
                               ("warmup_end", a.warmup_end), ("opt_config", a.opt_config)) if v is not None}
    if a.ignore_times:
        extra["ignore_times"] = True
    args = model_args(a, **extra)
    trainer = Trainer(args, device=dev, world=world, rank=rank, total_steps=a.steps, seed=a.seed,
                      sharded=a.sharded, accum_steps=a.accum_steps, grad_wire_dtype=a.grad_wire_dtype,
                      dp_impl=a.dp_impl, context_parallel=a.context_parallel, tp=a.tp)
    # context parallelism: every rank draws the same batch and keeps its segment of it; tensor
    # parallelism: the ranks of one tp group draw the same batch (their dp rank's)
    drank, dworld = (0, 1) if a.context_parallel else (trainer.rank, trainer.world)
    tickers = a.tickers.split(",") if a.tickers else None
    dr = tuple(a.train_date_range.split(",")) if a.train_date_range else None
    days = load_days(a.data_dir, a.synthetic, args.n_messages + 1, a.seed + 1000 * drank, tickers, dr)
    ds = LobWindowDataset([d.msgs for d in days], [d.books for d in days], args.n_messages,
                          token_mode=args.token_mode)
    sampler = WindowSampler(len(ds), args.micro_bsz, world=1 if not a.data_dir else dworld,
                            rank=0 if not a.data_dir else drank, seed=a.seed)

    def batches():
        for idx in sampler:
            yield collate([ds[i] for i in idx])
    cfg = LoopConfig(steps=a.steps, log_every=a.log_every, save_every=a.save_every, ckpt_dir=a.ckpt_dir,
                     resume=not a.no_resume, watchdog_timeout=a.watchdog_timeout, time_limit_s=a.time_limit_s,
                     ckpt_format=a.ckpt_format,
                     config={k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool))})
    log = (lambda r: print(json.dumps(r), flush=True)) if rank == 0 else (lambda r: None)
    res = fit(trainer, batches(), cfg, log=log)
    log({"event": "finished", "steps": res.steps_done, "stopped": res.stopped, "last_loss": res.last_loss})
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0 if res.stopped != "nan" else 2


if __name__ == "__main__":
    raise SystemExit(main())
