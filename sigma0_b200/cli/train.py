"""Training runtime: one process per GPU (torchrun), optional flat config file.

    torchrun --nproc-per-node 8 -m sigma0_b200.cli train --preset 350m --data_dir <days> \
        --ckpt_dir <dir> --steps 10000 --dp_impl fused

``--config`` reads a flat ``key: value`` file (``include:`` supported); its
``env_*`` keys are exported to the environment and its plain keys override
argument defaults (the reference's launch configs work unchanged for the keys
both sides know).  Mirrors ``run/base_model/runtime/train.py:47-330``: every flag of
the reference's training runtime is accepted under its own name -- model and
optimizer hyperparameters go to the model namespace the registry and the ``Trainer``
read (``_REF_MODEL``); data, schedule, checkpoint, validation, profiler and distributed
flags map onto this runtime's loop and ``Trainer``; the few with nothing to act on here
are accepted and recorded (``_REF_NOOP``, with the reason in their help text).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

from .common import add_model_args, dist_env, load_days, model_args


def str2bool(v) -> bool:
    if isinstance(v, bool):
        return v
    s = str(v).strip().lower()
    if s in ("true", "1", "yes", "y", "t"):
        return True
    if s in ("false", "0", "no", "n", "f"):
        return False
    raise argparse.ArgumentTypeError(f"expected a boolean, got {v!r}")


# reference flags that set a model / optimizer hyperparameter: (name, type, help); passed
# to the model namespace when given
_REF_MODEL = [
    ("activation_fn", str, "full_glu, half_glu1, half_glu2 or gelu"),
    ("attention_max_cache_len", int, "attention KV-cache length for decoding"),
    ("batchnorm", str2bool, "BatchNorm instead of LayerNorm in the sequence layers"),
    ("bn_momentum", float, "BatchNorm running-average momentum"),
    ("bidirectional", str2bool, "S5: bidirectional scan"),
    ("block_counts", int, "NSA: selected blocks per query"),
    ("block_size", int, "NSA: compression block size"),
    ("blocks", int, "S5: number of eigenvalue blocks"),
    ("C_init", str, "S5: C initialisation"),
    ("clip_eigs", str2bool, "S5: clip eigenvalues"),
    ("conj_sym", str2bool, "S5: conjugate symmetry"),
    ("cosine_anneal", str2bool, "cosine decay after warmup (else a constant lr)"),
    ("d_ff", int, "transformer feed-forward width (0: 4 d_model)"),
    ("discretization", str, "S5: zoh or bilinear"),
    ("dt_global", str2bool, "S5: log_step in the regular optimizer group"),
    ("dt_max", float, "S5: largest initial step"),
    ("dt_min", float, "S5: smallest initial step"),
    ("dtype", str, "compute dtype: float32 or bfloat16"),
    ("gdn_chunk_size", int, "GDN/KDA chunk size"),
    ("gdn_expand_v", int, "GDN/KDA value expansion"),
    ("gdn_head_dim", int, "GDN/KDA head dimension"),
    ("gdn_num_heads", int, "GDN/KDA heads (default d_model / head_dim)"),
    ("gdn_use_conv", str2bool, "GDN/KDA short convolutions"),
    ("hybrid_attn_d_ff", int, "hybrid: attention-block feed-forward width"),
    ("hybrid_attn_heads", int, "hybrid: attention heads"),
    ("hybrid_attn_layers", str, "hybrid: comma-separated attention layer indices"),
    ("hybrid_attn_positional_encoding", str2bool, "hybrid: positional encoding in attention blocks"),
    ("lr_min", float, "floor of the cosine schedule"),
    ("mamba3_chunk_size", int, "Mamba3 SSD chunk size"),
    ("mamba3_d_state", int, "Mamba3 state size N"),
    ("mamba3_expand", int, "Mamba3 expansion"),
    ("mamba3_headdim", int, "Mamba3 head dimension P"),
    ("mamba3_rope_fraction", float, "Mamba3 fraction of the state rotated"),
    ("max_grad_norm", float, "global gradient-norm clip"),
    ("model_type", str, "ssm or an attention model type"),
    ("muon_lr", float, "Muon learning rate (opt_config muon)"),
    ("muon_wd", float, "Muon weight decay (default weight_decay)"),
    ("n_book_post_layers", int, "book encoder layers after the projection"),
    ("n_book_pre_layers", int, "book encoder layers before the projection"),
    ("n_heads", int, "attention heads"),
    ("n_message_layers", int, "message encoder layers"),
    ("p_dropout", float, "dropout"),
    ("pe_type", str, "rope or sinusoidal"),
    ("prenorm", str2bool, "pre-norm sequence layers"),
    ("remat", str2bool, "recompute layer activations in the backward pass"),
    ("rope_base", float, "rotary base"),
    ("ssm_size_base", int, "S5 state size"),
    ("ssm_type", str, "backbone name (alias of --architecture)"),
    ("use_book_data", str2bool, "condition on the order book"),
    ("window_size", int, "NSA sliding window"),
]

# reference flags with nothing to act on in this runtime: (name, type, reason)
_REF_NOOP = [
    ("USE_WANDB", str2bool, "accepted; metrics are JSON lines on stdout (no wandb in this image)"),
    ("wandb_project", str, "accepted; recorded in the checkpoint config"),
    ("wandb_entity", str, "accepted; recorded in the checkpoint config"),
    ("dataset", str, "accepted; the LOBSTER window dataset is the only one"),
    ("merging", str, "accepted; book and message streams are always concatenated (padded)"),
    ("use_simple_book", str2bool, "accepted; the book is the transformed L2 volume image"),
    ("book_transform", str2bool, "accepted; the book transform is always applied"),
    ("hierarchical_nobook", str2bool, "accepted; the no-book hierarchy is --use_book_data false"),
    ("mode", str, "accepted; the decoder reads every position (none)"),
    ("mamba3_use_triton", str2bool, "accepted; the kernels are chosen by --impl"),
    ("mamba3_use_cuda", str2bool, "accepted; the kernels are chosen by --impl"),
    ("use_flash", str2bool, "accepted; attention always runs the fused kernels on CUDA"),
    ("hybrid_attn_flash", str2bool, "accepted; attention always runs the fused kernels on CUDA"),
    ("num_devices", int, "accepted; the device count is WORLD_SIZE"),
    ("n_data_workers", int, "accepted; windows are encoded in the training process"),
    ("prefetch_factor", int, "accepted; the next batch is copied while the step runs"),
    ("debug_loading", str2bool, "accepted"),
    ("uniform_ticker_batches", str2bool, "accepted; windows are drawn uniformly over all days"),
    ("log_ce_tables", str2bool, "accepted; per-field CE is logged by the evaluation pipeline"),
]


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="sigma0-b200 training runtime")
    p.add_argument("--config", default=None)
    add_model_args(p)
    # data
    p.add_argument("--data_dir", default=None)
    p.add_argument("--dir_name", "--data_root", dest="data_dir_ref", default=None, help="alias of --data_dir")
    p.add_argument("--tickers", default=None, help="comma-separated")
    p.add_argument("--train_date_range", default=None, help="YYYY-MM-DD,YYYY-MM-DD")
    p.add_argument("--test_date_range", default=None, help="days held out for validation (YYYY-MM-DD,YYYY-MM-DD)")
    p.add_argument("--test_dir_name", default=None, help="directory of validation days")
    p.add_argument("--synthetic", type=int, default=8, help="synthetic days when no --data_dir")
    p.add_argument("--n_messages", "--msg_seq_len", dest="n_messages", type=int, default=None)
    p.add_argument("--micro_bsz", type=int, default=None)
    p.add_argument("--masking", default="none", choices=["none", "causal", "random", "last_pos"],
                   help="training mask (none: plain next-token prediction)")
    p.add_argument("--book_depth", type=int, default=500, help="price levels of the transformed book")
    p.add_argument("--book_ablation", default="real", choices=["real", "zero", "noise", "shuffle"])
    p.add_argument("--shuffle_train", type=str2bool, default=True)
    p.add_argument("--random_offsets_train", type=str2bool, default=False,
                   help="shift every day's windows by a random per-epoch offset")
    p.add_argument("--debug_overfit", type=str2bool, default=False, help="train on the first batch only")
    p.add_argument("--val_split", type=float, default=0.001, help="fraction of windows held out for validation")
    p.add_argument("--no_validation", action="store_true")
    p.add_argument("--skip_test_eval", action="store_true", help="no validation at the end of training")
    p.add_argument("--val_batches", type=int, default=8, help="batches per validation")
    # schedule
    p.add_argument("--steps", type=int, default=None, help="optimizer steps (default: epochs x batches per epoch)")
    p.add_argument("--epochs", type=int, default=None)
    p.add_argument("--curtail_epochs", type=int, default=None, help="stop after this many epochs")
    p.add_argument("--mini_epochs", type=int, default=None, help="validate this many times per epoch")
    p.add_argument("--max_train_batches", type=int, default=0, help="batches per epoch (0: all)")
    p.add_argument("--lr", "--ssm_lr_base", dest="lr", type=float, default=None, help="ssm_lr_base")
    p.add_argument("--lr_factor", type=float, default=None)
    p.add_argument("--weight_decay", type=float, default=None)
    p.add_argument("--warmup_end", type=float, default=None)
    p.add_argument("--opt_config", default=None)
    p.add_argument("--ignore_times", type=str2bool, nargs="?", const=True, default=False)
    p.add_argument("--early_stop_patience", type=int, default=0, help="validations without improvement (0: off)")
    p.add_argument("--lr_patience", type=int, default=0, help="validations before the lr drops (0: off)")
    p.add_argument("--reduce_factor", type=float, default=0.9)
    p.add_argument("--eval_every", type=int, default=0, help="validate every N steps (0: per mini-epoch)")
    # checkpoints
    p.add_argument("--ckpt_dir", default=None)
    p.add_argument("--save_every", "--checkpoint_every_n_steps", dest="save_every", default="0",
                   help="steps between checkpoints; 'auto' = a tenth of the run")
    p.add_argument("--ckpt_format", choices=["native", "orbax"], default="native",
                   help="flat-buffer checkpoints or the Orbax StandardSave (zarr v2) layout")
    p.add_argument("--no_resume", action="store_true")
    p.add_argument("--resume_from_step", type=int, default=None, help="resume from this step of --ckpt_dir")
    p.add_argument("--restore", default=None, help="initialise from another run's checkpoint directory")
    p.add_argument("--restore_step", type=int, default=None)
    p.add_argument("--partial_restore", action="store_true", help="parameters only (by Flax path)")
    p.add_argument("--restore_reset_schedule", type=str2bool, default=False)
    p.add_argument("--log_every", type=int, default=100)
    p.add_argument("--watchdog_timeout", type=float, default=900.0)
    p.add_argument("--time_limit_s", type=float, default=None)
    p.add_argument("--max_job_hours", type=float, default=None, help="wall-clock budget (hours)")
    p.add_argument("--save_before_timeout_minutes", type=float, default=None,
                   help="save this long before the time budget runs out")
    # profiling
    p.add_argument("--enable_profiler", type=str2bool, default=False, help="trace optimizer steps 2..20")
    p.add_argument("--profile_steps", default=None, help="trace window START,STOP (optimizer steps)")
    p.add_argument("--profile_dir", default="profile")
    p.add_argument("--nvtx", action="store_true", help="NVTX range around every step")
    # distributed
    p.add_argument("--dp_impl", choices=["nccl", "fused"], default="nccl")
    p.add_argument("--sharded", action="store_true")
    p.add_argument("--fsdp", action="store_true",
                   help="ZeRO-3: shard the fused layers' projection kernels, gather them per layer")
    p.add_argument("--grad_wire_dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--accum_steps", "--grad_accum_steps", dest="accum_steps", type=int, default=1)
    p.add_argument("--tp", "--tp_size", dest="tp", type=int, default=1,
                   help="tensor-parallel size: heads split over groups of --tp consecutive ranks, batch over the rest")
    p.add_argument("--context_parallel", action="store_true",
                   help="split every sequence over the ranks (message-aligned segments) instead of the batch")
    p.add_argument("--hierarchical", type=str2bool, default=True,
                   help="two-level gradient reduction when the job spans several nodes")
    p.add_argument("--gpus_per_node", type=int, default=None, help="default LOCAL_WORLD_SIZE")
    p.add_argument("--local_steps_k", type=int, default=10, help="DiLoCo / FedAvg inner steps")
    p.add_argument("--diloco_outer", default="none", choices=["none", "diloco", "fedavg"])
    p.add_argument("--diloco_outer_lr", type=float, default=0.7)
    p.add_argument("--diloco_outer_momentum", type=float, default=0.9)
    p.add_argument("--seed", "--jax_seed", dest="seed", type=int, default=0)
    for name, typ, hlp in _REF_MODEL:
        if not any(name == a.dest for a in p._actions):
            p.add_argument(f"--{name}", type=typ, default=None, help=hlp)
    for name, typ, hlp in _REF_NOOP:
        p.add_argument(f"--{name}", type=typ, default=None, help=hlp)
    return p


def parse(argv=None):
    p = build_parser()
    a = p.parse_args(argv)
    if a.config:
        from ..utils.config import coerce, env_from_config, read_flat_config
        cfg = read_flat_config(a.config)
        env_from_config(cfg, apply=True)
        explicit = {x.split("=")[0].lstrip("-") for x in (argv if argv is not None else sys.argv[1:])
                    if x.startswith("--")}
        dests = {o.lstrip("-"): act.dest for act in p._actions for o in act.option_strings}
        for k, v in cfg.items():
            dest = dests.get(k)
            if dest is not None and k not in explicit and not k.startswith("env_"):
                setattr(a, dest, coerce(v))
    if a.data_dir is None and a.data_dir_ref:
        a.data_dir = a.data_dir_ref
    return a


def _ref_model_extra(a) -> dict:
    out = {}
    for name, _, _ in _REF_MODEL:
        v = getattr(a, name, None)
        if v is not None:
            out[name] = v
    if "ssm_type" in out and a.architecture is None:
        a.architecture = out["ssm_type"]
    return out


def _nodes(world: int, gpus_per_node) -> int:
    gpn = gpus_per_node or int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    return max(1, world // max(gpn, 1))


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
    extra.update(_ref_model_extra(a))
    args = model_args(a, **extra)

    # data: training days and held-out validation windows
    diloco = a.diloco_outer != "none" and world > 1
    cp = a.context_parallel and world > 1
    tickers = a.tickers.split(",") if a.tickers else None
    dr = tuple(a.train_date_range.split(",")) if a.train_date_range else None
    mask = {"none": "no_mask", "last_pos": "inference"}.get(a.masking, a.masking)
    ds_kw = dict(token_mode=args.token_mode, book_depth=a.book_depth, book_ablation=a.book_ablation,
                 use_book_data=bool(getattr(args, "use_book_data", True)), mask=mask, seed=a.seed,
                 random_offsets=a.random_offsets_train)
    # context parallelism: every rank draws the same batch and keeps its segment of it; tensor
    # parallelism: the ranks of one tp group draw the same batch (their dp rank's)
    tp = max(1, a.tp)
    drank, dworld = (0, 1) if cp else (rank // tp, world // tp)
    days = load_days(a.data_dir, a.synthetic, args.n_messages + 1, a.seed + 1000 * drank, tickers, dr)
    ds = LobWindowDataset([d.msgs for d in days], [d.books for d in days], args.n_messages, **ds_kw)
    val_ds, val_idx = None, None
    if not a.no_validation:
        if a.test_dir_name or a.test_date_range:
            tdr = tuple(a.test_date_range.split(",")) if a.test_date_range else None
            vdays = load_days(a.test_dir_name or a.data_dir, a.synthetic, args.n_messages + 1,
                              a.seed + 7919, tickers, tdr)
            val_ds = LobWindowDataset([d.msgs for d in vdays], [d.books for d in vdays], args.n_messages,
                                      **dict(ds_kw, random_offsets=False))
            val_idx = list(range(len(val_ds)))
        elif a.val_split > 0 and args.micro_bsz <= int(round(a.val_split * len(ds))) <= len(ds) - args.micro_bsz:
            # a held-out split only when it covers at least one batch and leaves one to train on
            n_val = int(round(a.val_split * len(ds)))
            perm = np.random.default_rng(a.seed + 17).permutation(len(ds))
            val_idx, train_idx = perm[:n_val].tolist(), np.sort(perm[n_val:])
            val_ds = ds
            ds = torch.utils.data.Subset(ds, train_idx.tolist())
    sampler = WindowSampler(len(ds), args.micro_bsz, world=1 if not a.data_dir else dworld,
                            rank=0 if not a.data_dir else drank, seed=a.seed, shuffle=a.shuffle_train)
    spe = max(sampler.steps_per_epoch(), 1)
    if a.max_train_batches:
        spe = min(spe, a.max_train_batches)
    if a.steps is not None:
        steps = a.steps
    else:
        epochs = a.epochs if a.epochs is not None else (100 if a.data_dir else max(1, -(-1000 // spe)))
        if a.curtail_epochs is not None:
            epochs = min(epochs, a.curtail_epochs)
        steps = epochs * spe
    save_every = max(steps // 10, 1) if str(a.save_every) == "auto" else int(a.save_every)

    hier = bool(a.hierarchical) and world > 1 and tp == 1 and not cp and not diloco and not a.sharded \
        and not a.fsdp and a.dp_impl == "nccl" and _nodes(world, a.gpus_per_node) > 1
    trainer = Trainer(args, device=dev, world=1 if diloco else world, rank=0 if diloco else rank,
                      total_steps=steps, seed=a.seed, sharded=a.sharded, accum_steps=a.accum_steps,
                      grad_wire_dtype=a.grad_wire_dtype, dp_impl=a.dp_impl, context_parallel=a.context_parallel,
                      tp=a.tp, hierarchical=hier, gpus_per_node=a.gpus_per_node, fsdp=a.fsdp)
    if diloco:
        from ..train.diloco import DiLoCo
        outer = DiLoCo(trainer, inner_steps=a.local_steps_k, outer_lr=a.diloco_outer_lr,
                       outer_momentum=a.diloco_outer_momentum, mode=a.diloco_outer)
        inner_step = trainer.step_device
        trainer.step_device = lambda *b: _diloco_step(outer, inner_step, b)

    base = ds.dataset if isinstance(ds, torch.utils.data.Subset) else ds

    def batches():
        """``spe`` batches per epoch from the sampler's per-epoch permutation (the loop skips
        the batches a resumed run has already consumed)."""
        if a.debug_overfit:
            first = collate([ds[i] for i in next(iter(sampler))])
            while True:
                yield first
        ep = 0
        while True:
            if hasattr(base, "set_epoch"):
                base.set_epoch(ep)
            idx = sampler.epoch_indices(ep)
            n = 0
            for k in range(spe):
                chunk = idx[k * args.micro_bsz:(k + 1) * args.micro_bsz]
                if len(chunk) < args.micro_bsz:
                    break
                yield collate([ds[i] for i in chunk.tolist()])
                n += 1
            if n == 0:
                raise RuntimeError(f"{len(idx)} training windows on this rank: fewer than one batch of "
                                   f"{args.micro_bsz}")
            ep += 1

    val_fn = None
    if val_ds is not None and val_idx:
        vb = args.micro_bsz
        nb = max(1, min(a.val_batches, len(val_idx) // vb))

        def val_fn():
            for k in range(nb):
                yield collate([val_ds[i] for i in val_idx[k * vb:(k + 1) * vb]])
    eval_every = a.eval_every or (max(spe // a.mini_epochs, 1) if a.mini_epochs else spe)
    prof = None
    if a.profile_steps:
        s0, s1 = (int(x) for x in a.profile_steps.split(","))
        prof = (s0, s1)
    elif a.enable_profiler:
        prof = (2, 20)
    time_limit = a.time_limit_s if a.time_limit_s is not None else \
        (a.max_job_hours * 3600.0 if a.max_job_hours is not None else None)
    cfg = LoopConfig(steps=steps, log_every=a.log_every, save_every=save_every, ckpt_dir=a.ckpt_dir,
                     resume=not a.no_resume, watchdog_timeout=a.watchdog_timeout, time_limit_s=time_limit,
                     save_margin_s=(a.save_before_timeout_minutes * 60.0 if a.save_before_timeout_minutes is not None
                                    else 300.0),
                     ckpt_format=a.ckpt_format, profile_steps=prof, profile_dir=a.profile_dir, nvtx=a.nvtx,
                     eval_every=eval_every if val_fn is not None else 0,
                     early_stop_patience=a.early_stop_patience, lr_patience=a.lr_patience,
                     reduce_factor=a.reduce_factor, resume_step=a.resume_from_step, restore_dir=a.restore,
                     restore_step=a.restore_step, partial_restore=a.partial_restore,
                     reset_schedule=a.restore_reset_schedule,
                     config={k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool))})
    log = (lambda r: print(json.dumps(r), flush=True)) if rank == 0 else (lambda r: None)
    res = fit(trainer, batches(), cfg, log=log,
              val_batches=None if (val_fn is None or a.skip_test_eval and not cfg.eval_every) else val_fn)
    log({"event": "finished", "steps": res.steps_done, "stopped": res.stopped, "last_loss": res.last_loss,
         "best_val_loss": res.best_val, "trace": res.trace_path})
    if a.ckpt_dir and rank == 0:
        # how the run ended, for a supervising launcher (torchrun reports any failure as exit 1)
        with open(os.path.join(a.ckpt_dir, "run_status.json"), "w") as f:
            json.dump({"stopped": res.stopped, "steps": res.steps_done, "last_loss": res.last_loss}, f)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0 if res.stopped != "nan" else 2


def _diloco_step(outer, inner_step, batch):
    """One inner step; every ``local_steps_k`` of them the outer synchronisation."""
    loss = inner_step(*batch)
    outer.inner += 1
    if outer.inner % outer.H == 0:
        outer.outer_step()
    return loss


if __name__ == "__main__":
    raise SystemExit(main())
