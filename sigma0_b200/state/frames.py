"""Wall-clock frames: event-level book states forward-filled onto a uniform grid.

The state model treats the book like video: one frame every ``interval_ns`` of
market time (1 ms by default), whatever the message rate.  A frame is the book
after the last event at or before its grid time; ``events_per_frame`` counts the
events folded into each frame (the information the fixed clock discards).

Input contract (the reference's ``state/frames.py:40-110`` and the wide-book npy
files): 3 metadata columns ``[delta_mid, time_s, time_ns]`` and then 4 columns per
level ``[ask_p, ask_s, bid_p, bid_s]``.  The grid starts at the first multiple of
``interval_ns`` at or after the first event, so every frame has a defined state,
and ends at the last event.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

META_COLS = 3
DEFAULT_INTERVAL_NS = 1_000_000


def absolute_time_ns(wide: np.ndarray) -> np.ndarray:
    """int64 nanoseconds after midnight from the (time_s, time_ns) metadata columns."""
    w = np.asarray(wide)
    if w.ndim != 2 or w.shape[1] <= META_COLS:
        raise ValueError(f"expected an (N, >{META_COLS}) wide-book array, got {w.shape}")
    return w[:, 1].astype(np.int64) * 1_000_000_000 + w[:, 2].astype(np.int64)


@dataclass
class FrameSeries:
    frames: np.ndarray            # (T, 4L) float32 book columns
    times_ns: np.ndarray          # (T,) grid times
    events_per_frame: np.ndarray  # (T,) events folded into each frame
    interval_ns: int

    @property
    def horizon_ns(self) -> int:
        return len(self.frames) * self.interval_ns


def resample_events(times_ns, states, interval_ns: int = DEFAULT_INTERVAL_NS) -> FrameSeries:
    """Forward-fill per-event states onto the ``interval_ns`` grid."""
    if interval_ns <= 0:
        raise ValueError("interval_ns must be positive")
    t = np.asarray(times_ns, dtype=np.int64)
    st = np.asarray(states)
    if t.ndim != 1 or t.size == 0:
        raise ValueError("times_ns must be a non-empty 1-D array")
    if st.shape[0] != t.shape[0]:
        raise ValueError("times_ns and states have different lengths")
    if (np.diff(t) < 0).any():
        raise ValueError("event times must be non-decreasing")
    first = ((t[0] + interval_ns - 1) // interval_ns) * interval_ns
    n = max(int((t[-1] - first) // interval_ns) + 1, 1)
    grid = first + interval_ns * np.arange(n, dtype=np.int64)
    upto = np.searchsorted(t, grid, side="right")          # events at or before each grid time
    frames = st[upto - 1].astype(np.float32)
    counts = np.diff(np.concatenate([[0], upto])).astype(np.int64)
    return FrameSeries(frames, grid, counts, int(interval_ns))


def resample_wide_book(wide: np.ndarray, interval_ns: int = DEFAULT_INTERVAL_NS) -> FrameSeries:
    """A wide-book day -> frames of its book columns (metadata used for the clock only)."""
    w = np.asarray(wide)
    book = w[:, META_COLS:]
    if book.shape[1] % 4:
        raise ValueError(f"book width must be divisible by 4, found {book.shape[1]}")
    return resample_events(absolute_time_ns(w), book, interval_ns)


def resample_frames(books: np.ndarray, interval_ns: int = DEFAULT_INTERVAL_NS,
                    n_frames: Optional[int] = None) -> Tuple[np.ndarray, np.ndarray]:
    """(frames, events_per_frame) of a wide-book array, optionally cut to ``n_frames``."""
    fs = resample_wide_book(books, interval_ns)
    if n_frames is not None:
        return fs.frames[:n_frames].astype(np.float64), fs.events_per_frame[:n_frames]
    return fs.frames.astype(np.float64), fs.events_per_frame
