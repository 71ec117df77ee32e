"""Shared CLI plumbing: rank discovery, model/preset arguments, data windows."""
from __future__ import annotations

import argparse
import os
from typing import Optional

import numpy as np
import torch


def add_model_args(p: argparse.ArgumentParser) -> None:
    p.add_argument("--preset", default="350m", help="model preset (smoke, 75m, 350m)")
    p.add_argument("--architecture", default=None, help="backbone name; must match the checkpoint when restoring")
    p.add_argument("--token_mode", default=None,
                   help="22tok/23tok/24tok/26tok, or 1tok (the one-position-per-message model; default: the preset's)")
    p.add_argument("--n_layers", type=int, default=None)
    p.add_argument("--d_model", type=int, default=None)
    p.add_argument("--impl", default=None, help="cuda (kernels) or torch (reference path)")


def model_args(a: argparse.Namespace, **extra):
    from ..models import preset_args
    kw = {k: v for k, v in (("architecture", a.architecture), ("token_mode", a.token_mode),
                            ("n_layers", a.n_layers), ("d_model", a.d_model)) if v is not None}
    kw["impl"] = a.impl or ("cuda" if torch.cuda.is_available() else "torch")
    kw.update(extra)
    if kw.get("token_mode"):
        from ..encoding import get_tokenizer
        from ..encoding.tok1 import encoding_mode
        tok = get_tokenizer(encoding_mode(kw["token_mode"]))
        kw.setdefault("msg_len", 1 if kw["token_mode"] == "1tok" else tok.MSG_LEN)
    return preset_args(a.preset, **kw)


def dist_env():
    """(rank, world, local_rank) from torchrun's environment (1 process when absent)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_days(data_dir: Optional[str], synthetic: int, n_msgs: int, seed: int, tickers=None, date_range=None):
    """Day arrays from ``data_dir`` (``*_message.npy`` / ``*_book.npy``) or synthetic days."""
    from ..data.lobster import MappedLobDay, resolve_day_files
    from ..data.masks import load_npy
    if data_dir:
        files = resolve_day_files(data_dir, tickers, date_range)
        if not files:
            raise FileNotFoundError(f"no *_message.npy / *_book.npy day files under {data_dir}")
        # memory-mapped: a window's rows are read when it is sampled, not at start-up
        return [MappedLobDay(load_npy(mf), load_npy(bf)) for mf, bf in files]
    from ..data.synthetic import make_sequences
    return make_sequences(synthetic, n_msgs, seed=seed)
