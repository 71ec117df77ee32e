"""State-model data windows, pretraining step, checkpoints and CLI.

Pipeline (the reference's ``state/dataset.py`` and ``state/train.py``):
wide-book day -> ``frames.resample_wide_book`` -> ``representation.encode_frames``
-> ``ChartNormalizer`` (fitted on the training days, stored in every checkpoint)
-> ``FrameWindowDataset`` windows of ``seq_len`` frames -> conditional flow matching
where every sample draws its own context length ``ctx ~ U{0..max_ctx}`` and the
loss counts generated frames only (a given frame's velocity is recoverable from its
own clean value).

Checkpoints: ``ckpt_<step>.pt`` (model, optimiser, normaliser, config) plus a
``latest_checkpoint.json`` pointer replaced atomically; resume follows the pointer.

    python -m sigma0_b200.state.train --data day1_book.npy day2_book.npy --out runs/state
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import tempfile
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset

from .dit import FrameDiT, FrameDiTConfig, bind_condition
from .flow import fm_loss, interpolate, velocity_target
from .frames import DEFAULT_INTERVAL_NS, FrameSeries, resample_wide_book
from .representation import ChartNormalizer, chart_channels, encode_frames


@dataclass
class EncodedDay:
    chart: np.ndarray        # (T, C) normalised chart frames
    anchor_mid: float
    interval_ns: int


def encode_series(series: FrameSeries, normalizer: Optional[ChartNormalizer], min_gap: float = 1.0,
                  with_activity: bool = False) -> EncodedDay:
    chart, anchor = encode_frames(series.frames, series.events_per_frame if with_activity else None, min_gap)
    if normalizer is not None:
        chart = normalizer.normalize(chart)
    return EncodedDay(chart, anchor, series.interval_ns)


def load_wide_book_day(path: str, interval_ns: int = DEFAULT_INTERVAL_NS) -> FrameSeries:
    return resample_wide_book(np.asarray(np.load(path, mmap_mode="r")), interval_ns)


def fit_normalizer(series: Sequence[FrameSeries], min_gap: float = 1.0,
                   with_activity: bool = False) -> ChartNormalizer:
    charts = [encode_frames(s.frames, s.events_per_frame if with_activity else None, min_gap)[0] for s in series]
    return ChartNormalizer.fit(np.concatenate(charts, 0))


class FrameWindowDataset(Dataset):
    """(window (seq_len, C) float32, anchor_mid) over strided windows of encoded days."""

    def __init__(self, days: Sequence[EncodedDay], seq_len: int, stride: Optional[int] = None):
        if seq_len < 2:
            raise ValueError("seq_len must be >= 2")
        stride = seq_len if stride is None else stride
        if stride < 1:
            raise ValueError("stride must be >= 1")
        self.days, self.seq_len = list(days), seq_len
        self.index = [(d, s) for d, day in enumerate(self.days)
                      for s in range(0, len(day.chart) - seq_len + 1, stride)]
        if not self.index:
            raise ValueError(f"no {seq_len}-frame window fits the days "
                             f"(lengths {[len(d.chart) for d in self.days]})")

    def __len__(self):
        return len(self.index)

    def __getitem__(self, i):
        d, s = self.index[i]
        day = self.days[d]
        return torch.from_numpy(np.array(day.chart[s:s + self.seq_len])), float(day.anchor_mid)


def sample_context_masks(batch: int, seq_len: int, max_ctx: int, device=None, generator=None) -> torch.Tensor:
    """obs_mask (B, L): 1 on a per-sample prefix of length ctx_i ~ U{0..max_ctx}."""
    if not 0 <= max_ctx < seq_len:
        raise ValueError("need 0 <= max_ctx < seq_len")
    ctx = torch.randint(0, max_ctx + 1, (batch,), device=device, generator=generator)
    return (torch.arange(seq_len, device=device)[None] < ctx[:, None]).float()


def pretrain_step(model: FrameDiT, x0: torch.Tensor, max_ctx: int, generator=None) -> dict:
    """Conditional flow-matching loss on clean windows x0 (B, L, C)."""
    B, L, _ = x0.shape
    obs = sample_context_masks(B, L, max_ctx, x0.device, generator)
    fn = bind_condition(model, x0, obs)
    t = torch.rand(B, device=x0.device, generator=generator)
    eps = torch.randn(x0.shape, device=x0.device, generator=generator)
    loss = fm_loss(fn(interpolate(x0, eps, t), t), velocity_target(x0, eps), frame_mask=1.0 - obs)
    return {"loss": loss, "ctx_mean": obs.sum(1).mean()}


def save_checkpoint(out_dir: str, step: int, model: FrameDiT, opt, normalizer: Optional[ChartNormalizer],
                    cfg: FrameDiTConfig) -> str:
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, f"ckpt_{step:08d}.pt")
    torch.save({"step": step, "model": model.state_dict(),
                "optimizer": None if opt is None else opt.state_dict(),
                "normalizer": None if normalizer is None else normalizer.state_dict(),
                "config": dataclasses.asdict(cfg)}, path)
    fd, tmp = tempfile.mkstemp(dir=out_dir, suffix=".json.tmp")
    with os.fdopen(fd, "w") as f:
        json.dump({"path": path, "step": step}, f)
    os.replace(tmp, os.path.join(out_dir, "latest_checkpoint.json"))
    return path


def load_checkpoint(out_dir: str, model: FrameDiT, opt=None) -> int:
    """Restore the checkpoint the pointer names; 0 when there is none."""
    ptr = os.path.join(out_dir, "latest_checkpoint.json")
    if not os.path.exists(ptr):
        return 0
    with open(ptr) as f:
        meta = json.load(f)
    st = torch.load(meta["path"], map_location="cpu", weights_only=False)
    model.load_state_dict(st["model"])
    if opt is not None and st.get("optimizer") is not None:
        opt.load_state_dict(st["optimizer"])
    return int(st["step"])


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description="state-model pretraining (conditional flow matching)")
    ap.add_argument("--data", nargs="+", required=True, help="wide-book .npy day files")
    ap.add_argument("--out", required=True)
    ap.add_argument("--interval_ns", type=int, default=DEFAULT_INTERVAL_NS)
    ap.add_argument("--seq_len", type=int, default=256)
    ap.add_argument("--max_ctx", type=int, default=128)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--hidden", type=int, default=128)
    ap.add_argument("--depth", type=int, default=4)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--with_activity", action="store_true")
    ap.add_argument("--min_gap", type=float, default=1.0)
    ap.add_argument("--save_every", type=int, default=500)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    torch.manual_seed(a.seed)
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    series = [load_wide_book_day(p, a.interval_ns) for p in a.data]
    norm = fit_normalizer(series, a.min_gap, a.with_activity)
    days = [encode_series(s, norm, a.min_gap, a.with_activity) for s in series]
    ds = FrameWindowDataset(days, a.seq_len)
    levels = series[0].frames.shape[1] // 4
    cfg = FrameDiTConfig(channels=chart_channels(levels, a.with_activity), hidden=a.hidden, depth=a.depth,
                         heads=a.heads, max_seq_len=max(a.seq_len, 16))
    model = FrameDiT(cfg).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=a.lr)
    step = load_checkpoint(a.out, model, opt)
    dl = DataLoader(ds, batch_size=a.batch, shuffle=True, drop_last=len(ds) >= a.batch)
    while step < a.steps:
        for x0, _ in dl:
            out = pretrain_step(model, x0.to(dev), a.max_ctx)
            opt.zero_grad(set_to_none=True)
            out["loss"].backward()
            opt.step()
            step += 1
            if step % 50 == 0:
                print(json.dumps({"step": step, "loss": float(out["loss"])}), flush=True)
            if step % a.save_every == 0 or step == a.steps:
                save_checkpoint(a.out, step, model, opt, norm, cfg)
            if step >= a.steps:
                break


if __name__ == "__main__":
    main()
