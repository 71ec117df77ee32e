"""Cross-entropy by message position and field (the reference's
``run/base_model/evaluate_ce_by_position.py``): mean CE of each of the MSG_LEN
token positions over evaluation windows, and per field.

    python -m sigma0_b200.eval.ce_by_position --preset 75m --ckpt_path <dir> --data_dir <days>
"""
from __future__ import annotations

import argparse
import json
from typing import Dict

import numpy as np
import torch


def ce_by_position(model, batches, tokenizer) -> Dict:
    L = tokenizer.MSG_LEN
    tot, n = np.zeros(L), 0
    dev = next(model.parameters()).device
    with torch.no_grad():
        for tokens, labels, book in batches:
            logp = model(tokens.to(dev), book.to(dev) if book is not None else None)
            nll = -logp.gather(-1, labels.to(dev)[..., None])[..., 0].float().cpu().numpy()
            B, T = nll.shape
            tot += nll.reshape(B, T // L, L).sum((0, 1))
            n += B * (T // L)
    pos = tot / max(n, 1)
    starts = np.concatenate([[0], np.cumsum(tokenizer.TOK_LENS)])
    fields = {f: float(pos[starts[i]:starts[i + 1]].mean()) for i, f in enumerate(tokenizer.FIELDS)}
    return {"n_messages": n, "by_position": pos.tolist(), "by_field": fields, "mean": float(pos.mean())}


def main(argv=None):
    from ..cli.common import add_model_args, load_days, model_args
    from ..data import LobWindowDataset, collate
    from ..encoding import get_tokenizer
    from ..models import build_model
    p = argparse.ArgumentParser()
    add_model_args(p)
    p.add_argument("--ckpt_path", default=None)
    p.add_argument("--checkpoint_step", type=int, default=None)
    p.add_argument("--data_dir", default=None)
    p.add_argument("--synthetic", type=int, default=2)
    p.add_argument("--n_messages", type=int, default=100)
    p.add_argument("--batch_size", type=int, default=2)
    p.add_argument("--max_batches", type=int, default=10)
    a = p.parse_args(argv)
    args = model_args(a, n_messages=a.n_messages)
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    if a.ckpt_path:
        from ..ckpt import CheckpointManager
        from ..train.trainer import Trainer
        tr = Trainer(args, device=dev)
        CheckpointManager(a.ckpt_path).restore(tr, step=a.checkpoint_step, params_only=True)
        model = tr.model
    else:
        model = build_model(args).to(dev)
    model.eval()
    days = load_days(a.data_dir, a.synthetic, a.n_messages + 1, 0)
    ds = LobWindowDataset([d.msgs for d in days], [d.books for d in days], a.n_messages, token_mode=args.token_mode)
    batches = (collate([ds[j] for j in range(i, min(i + a.batch_size, len(ds)))])
               for i in range(0, min(len(ds), a.batch_size * a.max_batches), a.batch_size))
    print(json.dumps(ce_by_position(model, batches, get_tokenizer(args.token_mode))))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
