"""Masking objectives and book ablations for message windows.

A window is an (n_messages, MSG_LEN) array of token ids.  The objectives of the
reference's ``LOBSTER_Dataset`` (``data/lobster_dataloader.py:567-870``), own code:

* ``no_mask`` -- next-token prediction over the flattened window: input is the
  stream shifted right behind a START token, the label is the stream (training
  default); ``no_mask_1tok`` shifts by one message row (1-token-per-message
  encoding); ``inference_mask`` prepends START and returns no label.
* ``masking_fn(tok, random_msg_idxs | random_fields, randomize_message)`` --
  one token of one message (a random message, or the last) becomes MASK and is the
  label; candidate positions are given directly or as whole fields.
* ``random_mask`` -- in the last message, a random non-empty subset of positions
  is hidden (HIDDEN) and one of them is masked (MASK, the label); the absolute-time
  field is excluded and hidden whenever part of delta_t is.
* ``causal_mask`` -- in the last message one token of a chosen field is masked,
  the rest of that field and a set of other fields are hidden; ``selector`` picks
  the fields: ``sequential_no_time`` (default: every field after the masked one,
  never the time fields), ``sequential``, ``random`` or ``unconditional``.
* ``ablate_books`` -- ``real`` / ``zero`` / ``noise`` (N(0, 0.15) after the
  three leading columns) / ``shuffle`` (message order permuted), seeded per window.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from ..encoding import HIDDEN_TOK, MASK_TOK, START_TOK


def field_slice(tok, field_i: int) -> Tuple[int, int]:
    """[start, end) token positions of field ``field_i`` inside one message."""
    start = int(np.concatenate([[0], np.cumsum(tok.TOK_LENS)])[field_i])
    return start, start + int(tok.TOK_LENS[field_i])


def no_mask(seq: np.ndarray, books=None):
    flat = np.asarray(seq).reshape(-1)
    return (np.concatenate([[START_TOK], flat[:-1]]), books), flat.copy()


def no_mask_1tok(seq: np.ndarray, books=None):
    s = np.asarray(seq)
    start = np.full((1, s.shape[1]), START_TOK, dtype=s.dtype)
    return (np.concatenate([start, s[:-1]], 0), books), s.copy()


def inference_mask(seq: np.ndarray, books=None):
    return (np.concatenate([[START_TOK], np.asarray(seq).reshape(-1)]), books), np.array(0)


def masking_fn(tok, *, random_msg_idxs: Optional[Sequence[int]] = None,
               random_fields: Optional[Sequence[str]] = None, randomize_message: bool = True) -> Callable:
    """fn(seq, rng) -> (masked seq, label) masking one token."""
    if (random_msg_idxs is None) == (random_fields is None):
        raise ValueError("give exactly one of random_msg_idxs and random_fields")
    if random_fields is not None:
        pos: List[int] = []
        for f in random_fields:
            a, b = field_slice(tok, tok.FIELDS.index(f))
            pos += list(range(a, b))
    else:
        pos = [int(i) for i in random_msg_idxs]

    def fn(seq, rng):
        s = np.array(seq, copy=True)
        m = int(rng.integers(0, s.shape[0])) if randomize_message else s.shape[0] - 1
        t = pos[0] if len(pos) == 1 else int(rng.choice(pos))
        y = s[m, t]
        s[m, t] = MASK_TOK
        return s, y

    return fn


def random_mask(tok, seq, rng, exclude_time: bool = True):
    s = np.array(seq, copy=True)
    L = tok.MSG_LEN
    if exclude_time:
        t0, t1 = tok.TIME_START_I, tok.TIME_END_I + 1
        cand = [i for i in range(L) if not t0 <= i < t1]
    else:
        t0 = t1 = 0
        cand = list(range(L))
    n_hid = int(rng.integers(1, len(cand) + 1))
    hid = sorted(int(i) for i in rng.choice(cand, n_hid, replace=False))
    msk = int(rng.choice(hid))
    hid.remove(msk)
    if exclude_time:
        a, b = field_slice(tok, tok.FIELDS.index("delta_t_s"))
        c, d = field_slice(tok, tok.FIELDS.index("delta_t_ns"))
        if any(a <= i < b or c <= i < d for i in hid + [msk]):
            hid += list(range(t0, t1))                # partly hidden delta_t: hide the time too
    y = s[-1, msk]
    s[-1, msk] = MASK_TOK
    s[-1, hid] = HIDDEN_TOK
    return s, y


def _select_fields(tok, rng, selector: str):
    """(hidden field indices, masked field index)."""
    F = len(tok.FIELDS)
    if selector == "random":
        sel = sorted(int(i) for i in rng.choice(F, int(rng.integers(1, F + 1)), replace=False))
        m = int(rng.choice(sel))
        return [f for f in sel if f != m], m
    if selector == "unconditional":
        m = int(rng.integers(0, F))
        return [f for f in range(F) if f != m], m
    if selector == "sequential":
        m = int(rng.integers(0, F))
        return list(range(m + 1, F)), m
    if selector == "sequential_no_time":
        ts, tn = tok.FIELDS.index("time_s"), tok.FIELDS.index("time_ns")
        others = [f for f in range(F) if f not in (ts, tn)]
        m = others[int(rng.integers(0, len(others)))]
        return list(range(m + 1, F)), m
    raise ValueError(f"unknown causal-mask selector {selector!r}")


def causal_mask(tok, seq, rng, selector: str = "sequential_no_time"):
    s = np.array(seq, copy=True)
    hidden, m = _select_fields(tok, rng, selector)
    a, b = field_slice(tok, m)
    t = int(rng.integers(a, b))
    y = s[-1, t]
    s[-1, t] = MASK_TOK
    s[-1, t + 1:b] = HIDDEN_TOK
    for f in hidden:
        fa, fb = field_slice(tok, f)
        s[-1, fa:fb] = HIDDEN_TOK
    return s, y


def ablate_books(book: np.ndarray, mode: str, seed: Sequence[int]) -> np.ndarray:
    if mode == "real":
        return book
    if mode == "zero":
        return np.zeros_like(book)
    rng = np.random.default_rng(list(seed))
    if mode == "noise":
        out = np.zeros_like(book)
        out[:, 3:] = rng.standard_normal((book.shape[0], book.shape[1] - 3)) * 0.15
        return out
    if mode == "shuffle":
        return book[rng.permutation(book.shape[0])]
    raise ValueError(f"unknown book ablation {mode!r}; use real, zero, noise or shuffle")


def load_npy(path: str, mmap_mode: Optional[str] = "r") -> np.ndarray:
    """``.npy`` (memory-mapped) or ``.npy.zst``: the plain file wins when both exist; a
    ``.npy.zst`` is decompressed with the ``zstandard`` module, else the system libzstd."""
    plain = path[:-4] if path.endswith(".zst") else path
    import os
    if os.path.exists(plain):
        return np.load(plain, mmap_mode=mmap_mode)
    zst = plain + ".zst"
    if not os.path.exists(zst):
        raise FileNotFoundError(plain)
    import io
    try:
        import zstandard
        with open(zst, "rb") as f:
            data = zstandard.ZstdDecompressor().stream_reader(f).read()
    except ImportError:                                # the system libzstd through ctypes
        from ..utils import zstd
        with open(zst, "rb") as f:
            data = zstd.decompress(f.read())
    return np.load(io.BytesIO(data))
