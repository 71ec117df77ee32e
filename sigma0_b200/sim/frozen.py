"""Frozen market-making episodes: one conditioning window, the background order flow one
world model generated for it and the forward mid-price curve a second model expects, kept
in one file so that every policy is scored against exactly the same market.

The reference's episode builder (``src/post_training/heuristic_learning/episode_builder.py:
126-253``) fixes the contract kept here:

* a background stream whose clock runs backwards cannot be replayed meaningfully, so it is
  rejected (``EpisodeError``), never repaired in place;
* the signal is a summary of J rollouts of the signal model from the same context, per
  horizon in messages: the mean mid and its 10% / 90% quantiles across rollouts (the
  model's own uncertainty, not estimation noise);
* an episode file is written once, atomically (write then rename), and an existing one is
  authoritative when a build resumes;
* the whole pipeline is gated by a replay check: the generated messages replayed from the
  conditioning book must reproduce the books the generator recorded.

Episodes are ``.npz`` files ``episode_<window>.npz``; the generation run layout is the one
``cli/infer.py`` writes (read with ``sim.divergence``).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import numpy as np

from .fidelity import compare_paths, mid_from_book, replay_stream


class EpisodeError(ValueError):
    pass


@dataclass(frozen=True)
class EpisodeSpec:
    window_id: int
    stock: str
    date: str
    background_seed: int
    signal_seeds: Tuple[int, ...]
    bg_checkpoint: str = ""          # pin names (``ckpt.pins``) of the two world models
    signal_checkpoint: str = ""


def stream_timing(msgs: np.ndarray) -> Dict[str, object]:
    """Clock and event-type summary of a message stream (engine rows, time in columns 6 / 7)."""
    m = np.asarray(msgs, np.int64)
    t = m[:, 6] * 1_000_000_000 + m[:, 7]
    dt = np.diff(t)
    types, counts = np.unique(m[:, 0], return_counts=True)
    return {"n_messages": int(len(m)), "span_s": float(t[-1] - t[0]) / 1e9 if len(t) > 1 else 0.0,
            "monotonic": bool((dt >= 0).all()), "n_negative_deltas": int((dt < 0).sum()),
            "min_delta_ns": int(dt.min()) if len(dt) else 0,
            "event_types": {int(a): int(b) for a, b in zip(types, counts)}}


def require_replayable(timing: Dict[str, object], source: str) -> None:
    if not timing["monotonic"]:
        raise EpisodeError(f"{source}: the clock runs backwards {timing['n_negative_deltas']} times "
                           f"(smallest step {timing['min_delta_ns']} ns); discard the window")


def signal_curve(rollout_books: Sequence[np.ndarray], horizons: Sequence[int]) -> Dict[str, np.ndarray]:
    """Forward mid curve of J rollouts (each an (n, 4L) book path after each generated
    message): at each horizon h (messages) the mean and the 10% / 90% quantiles of the mid
    after message h across rollouts; rollouts shorter than h contribute nothing there."""
    if not len(rollout_books):
        raise EpisodeError("the signal curve needs at least one rollout")
    hs = [int(h) for h in horizons]
    mids = [mid_from_book(np.asarray(b)) for b in rollout_books]
    arr = np.array([[m[h - 1] if 0 < h <= len(m) else np.nan for h in hs] for m in mids], np.float64)
    with np.errstate(invalid="ignore"):
        return {"horizons": np.asarray(hs, np.int32), "anchor_mid": np.float64(np.mean([m[0] for m in mids])),
                "mid_mean": np.nanmean(arr, 0), "mid_q10": np.nanquantile(arr, 0.10, 0),
                "mid_q90": np.nanquantile(arr, 0.90, 0), "n_rollouts": np.int32(len(mids))}


def build_episode(spec: EpisodeSpec, init_book: np.ndarray, background: np.ndarray,
                  signal: Dict[str, np.ndarray]) -> Dict[str, object]:
    timing = stream_timing(background)
    require_replayable(timing, f"window {spec.window_id}")
    ep = {"window_id": np.int32(spec.window_id), "stock": spec.stock, "date": spec.date,
          "init_book": np.asarray(init_book, np.int64), "background": np.asarray(background, np.int64),
          "background_timing": json.dumps(timing), "background_seed": np.int32(spec.background_seed),
          "signal_seeds": np.asarray(spec.signal_seeds, np.int32), "bg_checkpoint": spec.bg_checkpoint,
          "signal_checkpoint": spec.signal_checkpoint}
    ep.update({f"signal_{k}": v for k, v in signal.items()})
    return ep


def save_episode(ep: Dict[str, object], out_dir: str) -> str:
    """Write ``ep`` once (temporary file, then an atomic rename); an existing file wins."""
    os.makedirs(out_dir, exist_ok=True)
    final = os.path.join(out_dir, f"episode_{int(ep['window_id']):06d}.npz")
    if os.path.exists(final):
        return final
    tmp = final + ".tmp.npz"
    np.savez_compressed(tmp, **ep)
    os.replace(tmp, final)
    return final


def load_episode(path: str) -> Dict[str, object]:
    with np.load(path, allow_pickle=False) as z:
        ep = {k: z[k] for k in z.files}
    for k in ("stock", "date", "bg_checkpoint", "signal_checkpoint", "background_timing"):
        ep[k] = str(ep[k])
    ep["background_timing"] = json.loads(ep["background_timing"])
    return ep


def run_windows(root: str, stock: str, limit: int) -> List[Tuple[str, int]]:
    """Up to ``limit`` (date, index) pairs of generated windows in a run's ``data_gen``
    (the index is the dataset index of the conditioning window, so it is discovered)."""
    out: List[Tuple[str, int]] = []
    pre, mid, suf = f"{stock}_", "_message_real_id_", "_gen_id_0.csv"
    with os.scandir(os.path.join(root, "data_gen")) as it:
        for e in it:
            n = e.name
            if n.startswith(pre) and n.endswith(suf) and mid in n:
                date, rest = n[len(pre):].split(mid)
                out.append((date, int(rest[:-len(suf)])))
                if len(out) >= limit:
                    break
    return sorted(out)


def replay_gate(root: str, stock: str, n: int = 8) -> Dict[str, Dict[str, float]]:
    """The pipeline's consistency check: for up to ``n`` generated windows, replay the
    generated messages from the conditioning book and compare with the generator's own
    recorded books (an exact-mid fraction below 1 means the CSV round trip or the replay
    lost something, and every PnL built on it would be quietly wrong)."""
    from .divergence import read_books, read_messages, run_paths
    out = {}
    for date, i in run_windows(root, stock, n):
        p = run_paths(root, stock, date, i)
        init = read_books(p["cond_book"])[-1]
        books = read_books(p["gen_book"])
        path, rep = replay_stream(read_messages(p["gen_msg"]), init, books.shape[1] // 4)
        out[f"{date} #{i}"] = {**compare_paths(path, books), "clean": rep.clean}
    return out
