"""Generation runtime: condition on real windows, generate with the engine in the loop, write CSVs.

One process per GPU (torchrun); windows are split across ranks by interleaving
(window i goes to rank i % world) and every rank seeds with ``seed + rank``
(``run/base_model/runtime/inference.py:80-136,475-605``).  Output layout
(``docs/inference.md``):

    <save_dir>/data_cond/<stock>_<date>_message_real_id_<i>.csv     conditioning messages
    <save_dir>/data_cond/<stock>_<date>_orderbook_real_id_<i>.csv   N+1 book rows (incl. the opening one)
    <save_dir>/data_gen/<stock>_<date>_message_real_id_<i>_gen_id_0.csv
    <save_dir>/data_gen/<stock>_<date>_orderbook_real_id_<i>_gen_id_0.csv
    <save_dir>/data_gen/<stock>_<date>_provenance_real_id_<i>_gen_id_0.csv
    <save_dir>/data_real/<stock>_<date>_message_real_id_<i>.csv     the real continuation
    <save_dir>/data_real/<stock>_<date>_orderbook_real_id_<i>.csv
    <save_dir>/sample_indices_rank<k>.json

Messages use the LOBSTER layout ``time, event_type, order_id, size, price, direction``
(time = seconds.nanoseconds, direction -1/1).
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch

from .common import add_model_args, dist_env, load_days, model_args


def lobster_messages(raw: np.ndarray):
    """(n, 14) message rows -> LOBSTER message DataFrame."""
    import pandas as pd
    r = np.asarray(raw, dtype=np.int64)
    time = [f"{s}.{ns:09d}" for s, ns in zip(r[:, 8], r[:, 9])]
    return pd.DataFrame({"time": time, "event_type": r[:, 1], "order_id": r[:, 0], "size": r[:, 5],
                         "price": r[:, 3], "direction": np.where(r[:, 2] == 0, -1, 1)})


def parse(argv=None):
    p = argparse.ArgumentParser(description="sigma0-b200 generation runtime")
    add_model_args(p)
    p.add_argument("--ckpt_path", default=None)
    p.add_argument("--checkpoint_step", type=int, default=None)
    p.add_argument("--data_dir", default=None)
    p.add_argument("--synthetic", type=int, default=0, help="use N synthetic days instead of --data_dir")
    p.add_argument("--save_dir", required=True)
    p.add_argument("--stock", default="SYN")
    p.add_argument("--date", default="2000-01-01")
    p.add_argument("--n_sequences", type=int, default=8)
    p.add_argument("--window_starts_file", default=None,
                   help="JSON of explicit (file_idx, seq_start) windows (python -m sigma0_b200.eval.trade_anchors)")
    p.add_argument("--batch_size", type=int, default=8)
    p.add_argument("--n_cond_msgs", type=int, default=500)
    p.add_argument("--n_gen_msgs", type=int, default=100)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--sample_top_n", type=int, default=-1)
    p.add_argument("--no_graphs", action="store_true")
    p.add_argument("--inject_step", type=int, default=None)
    p.add_argument("--inject_event_type", type=int, default=4)
    p.add_argument("--inject_side", type=int, default=1)
    p.add_argument("--inject_qty", type=int, default=100)
    p.add_argument("--inject_price_offset_ticks", type=int, default=0)
    return p.parse_args(argv)


def main(argv=None):
    from ..data.book_transform import transform_books_numpy
    from ..encoding import START_TOK, get_tokenizer
    from ..infer import Generator
    from ..models import build_model
    a = parse(argv)
    rank, world, local = dist_env()
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    args = model_args(a)
    tok = get_tokenizer(args.token_mode)
    torch.manual_seed(a.seed + rank)
    model = build_model(args).to(dev).eval()
    if a.ckpt_path:
        from ..ckpt import CheckpointManager
        from ..train.trainer import Trainer
        tr = Trainer(args, device=dev)
        CheckpointManager(a.ckpt_path).restore(tr, step=a.checkpoint_step, params_only=True)
        model = tr.model.eval()
    need = a.n_cond_msgs + a.n_gen_msgs + 1
    days = load_days(a.data_dir, a.synthetic or a.n_sequences, need, a.seed)
    windows = []
    if a.window_starts_file:
        from ..data.lobster import resolve_day_files
        from ..eval.trade_anchors import load_window_starts
        files = [mf for mf, _ in resolve_day_files(a.data_dir)] if a.data_dir else None
        windows = load_window_starts(a.window_starts_file, files)
        for di, s in windows:
            if not (0 <= di < len(days) and 0 <= s and s + need <= min(days[di].msgs.shape[0] + 1, days[di].books.shape[0])):
                raise ValueError(f"window ({di}, {s}) does not fit its day")
    else:
        for di, d in enumerate(days):
            for s in range(0, d.msgs.shape[0] - need + 1, need):
                windows.append((di, s))
        windows = windows[:a.n_sequences]
    mine = [i for i in range(len(windows)) if i % world == rank]
    for sub in ("data_cond", "data_gen", "data_real"):
        os.makedirs(os.path.join(a.save_dir, sub), exist_ok=True)
    with open(os.path.join(a.save_dir, f"sample_indices_rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "world": world, "windows": [list(windows[i]) for i in mine]}, f)
    nc, ng = a.n_cond_msgs, a.n_gen_msgs
    inject = None
    if a.inject_step is not None:
        inject = {"step": a.inject_step, "event_type": a.inject_event_type, "side": a.inject_side,
                  "qty": a.inject_qty, "offset_ticks": a.inject_price_offset_ticks}
    pre = f"{a.stock}_{a.date}"
    for b0 in range(0, len(mine), a.batch_size):
        batch = mine[b0:b0 + a.batch_size]
        x, bk, last, l2s, em = [], [], [], [], []
        for i in batch:
            di, s = windows[i]
            d = days[di]
            t = tok.encode_msgs(d.msgs[s:s + nc]).reshape(-1)
            x.append(np.concatenate([[START_TOK], t[:-1]]))
            last.append(t[-1])
            bk.append(transform_books_numpy(d.books[s:s + nc]).astype(np.float32))
            l2s.append(d.books[s, 3:].astype(np.int64))
            em.append(d.engine_msgs[s:s + nc])
        gen = Generator(model, args.token_mode, top_n=a.sample_top_n, seed=a.seed + rank,
                        use_graphs=not a.no_graphs and dev.type == "cuda")
        gen.condition(torch.tensor(np.stack(x)), torch.tensor(np.stack(bk)), torch.tensor(last), np.stack(l2s),
                      np.stack(em), start_time=(int(days[windows[batch[0]][0]].books[windows[batch[0]][1], 1]), 0))
        out = gen.generate(ng, inject=inject)
        raw = out.raw.cpu().numpy()
        l2 = out.l2.cpu().numpy()
        prov = out.provenance.cpu().numpy()
        mids = out.mid.cpu().numpy()
        for j, i in enumerate(batch):
            di, s = windows[i]
            d = days[di]
            lobster_messages(d.msgs[s:s + nc]).to_csv(
                os.path.join(a.save_dir, "data_cond", f"{pre}_message_real_id_{i}.csv"), index=False)
            import pandas as pd
            cond_books = np.concatenate([d.books[s:s + nc, 3:], d.books[s + nc:s + nc + 1, 3:]]).astype(np.int64)
            pd.DataFrame(cond_books).to_csv(os.path.join(a.save_dir, "data_cond", f"{pre}_orderbook_real_id_{i}.csv"),
                                            index=False)
            lobster_messages(d.msgs[s + nc:s + nc + ng]).to_csv(
                os.path.join(a.save_dir, "data_real", f"{pre}_message_real_id_{i}.csv"), index=False)
            pd.DataFrame(d.books[s + nc + 1:s + nc + ng + 1, 3:].astype(np.int64)).to_csv(
                os.path.join(a.save_dir, "data_real", f"{pre}_orderbook_real_id_{i}.csv"), index=False)
            lobster_messages(raw[j]).to_csv(
                os.path.join(a.save_dir, "data_gen", f"{pre}_message_real_id_{i}_gen_id_0.csv"), index=False)
            pd.DataFrame(l2[j]).to_csv(
                os.path.join(a.save_dir, "data_gen", f"{pre}_orderbook_real_id_{i}_gen_id_0.csv"), index=False)
            pd.DataFrame({"provenance": prov[j], "mid_after": mids[j]}).to_csv(
                os.path.join(a.save_dir, "data_gen", f"{pre}_provenance_real_id_{i}_gen_id_0.csv"), index=False)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
