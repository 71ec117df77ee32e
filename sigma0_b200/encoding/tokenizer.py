"""Table-driven message tokenizers for the 22/23/24/26-token encodings.

One generic implementation covers every multi-token mode; a mode is a
``ModeSpec`` (vocabulary field order plus the per-field token layout).  The
resulting vocabularies and token ids match the reference tokenizers:

* 22tok: ``src/base_model/encoding/encoding_22tok.py:220-238`` (vocab 12012),
  ``TOK_LENS`` at ``:302``, ``encode_msg`` ``:94``, ``decode_msg`` ``:159``.
* 23tok: ``encoding_23tok.py:254-270`` (fused event_dir), ``TOK_LENS`` ``:335``.
* 24tok: ``encoding_24tok.py:295-311`` (base-100 size), ``TOK_LENS`` ``:376``.
* 26tok: ``encoding_26tok.py:269-286`` (base-1000 two-digit price),
  ``TOK_LENS`` ``:351``.

Raw message rows use the reference's 14-column preprocessed layout
(``encoding_22tok.py:251`` field names)::

    [order_id, event_type, direction, price_abs, price, size,
     delta_t_s, delta_t_ns, time_s, time_ns,
     price_ref, size_ref, time_s_ref, time_ns_ref]

Value -> token lookups reproduce the reference's binary search exactly,
including how it treats the special sentinels (the reference searches a
key table whose first four entries are not sorted; see ``_bsearch_left``).
Everything here is numpy and vectorised over messages.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

import numpy as np

NA_VAL = -9999
HIDDEN_VAL = -20000
MASK_VAL = -10000
START_VAL = -30000
SPECIAL_VALS = (MASK_VAL, HIDDEN_VAL, NA_VAL, START_VAL)

MASK_TOK, HIDDEN_TOK, NA_TOK, START_TOK = 0, 1, 2, 3
N_SPECIAL = 4

RAW_FIELDS = ("order_id", "event_type", "direction", "price_abs", "price",
              "size", "delta_t_s", "delta_t_ns", "time_s", "time_ns",
              "price_ref", "size_ref", "time_s_ref", "time_ns_ref")
RAW_I = {n: i for i, n in enumerate(RAW_FIELDS)}


def _bsearch_left(sorted_keys: np.ndarray, q: np.ndarray) -> np.ndarray:
    """Fixed-depth binary search, ``ceil(log2(n+1))`` halvings.

    This is the exact search the reference's ``encode``/``decode`` run
    (``encoding_22tok.py:17-27``): low=0, high=n; each level moves ``high`` to
    mid when ``q <= keys[mid]``.  Keys may be partially unsorted (the special
    sentinels sit first), so the result for a sentinel is whatever this search
    lands on -- reproduced here, not "fixed".
    """
    keys = np.asarray(sorted_keys)
    q = np.asarray(q)
    n = keys.shape[0]
    levels = int(np.ceil(np.log2(n + 1)))
    lo = np.zeros(q.shape, dtype=np.int64)
    hi = np.full(q.shape, n, dtype=np.int64)
    for _ in range(levels):
        mid = (lo + hi) // 2
        go_left = q <= keys[np.minimum(mid, n - 1)]
        lo = np.where(go_left, lo, mid)
        hi = np.where(go_left, mid, hi)
    return hi


@dataclass
class FieldCode:
    """Lookup tables for one vocabulary field (value <-> global token id)."""
    name: str
    values: np.ndarray          # real values, in vocabulary order
    keys: np.ndarray            # [MASK, HIDDEN, NA, START, *values]
    toks: np.ndarray            # [0, 1, 2, 3, offset + arange(len(values))]
    offset: int

    def encode(self, x: np.ndarray) -> np.ndarray:
        idx = _bsearch_left(self.keys, x)
        return self.toks[np.minimum(idx, len(self.toks) - 1)]

    def decode(self, t: np.ndarray) -> np.ndarray:
        idx = _bsearch_left(self.toks, t)
        return self.keys[np.minimum(idx, len(self.keys) - 1)]


class Vocabulary:
    """Global token ids: 4 specials, then each field's values in order."""

    MASK_TOK = MASK_TOK
    HIDDEN_TOK = HIDDEN_TOK
    NA_TOK = NA_TOK
    START_TOK = START_TOK

    def __init__(self, fields: Sequence[Tuple[str, Sequence[int]]]):
        self.counter = N_SPECIAL
        self.codes: Dict[str, FieldCode] = {}
        for name, vals in fields:
            vals = np.asarray(list(vals), dtype=np.int64)
            keys = np.concatenate([np.array(SPECIAL_VALS, dtype=np.int64), vals])
            toks = np.concatenate([np.arange(N_SPECIAL, dtype=np.int64),
                                   self.counter + np.arange(len(vals), dtype=np.int64)])
            self.codes[name] = FieldCode(name, vals, keys, toks, self.counter)
            self.counter += len(vals)
        # reference-style ENCODING dict: field -> (keys, toks)
        self.ENCODING = {n: (c.keys, c.toks) for n, c in self.codes.items()}

    def __len__(self) -> int:
        return self.counter

    def field_range(self, name: str) -> Tuple[int, int]:
        c = self.codes[name]
        return c.offset, c.offset + len(c.values)


# ---------------------------------------------------------------------------
# Mode specifications
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class ModeSpec:
    name: str
    vocab_fields: Tuple[Tuple[str, Tuple[int, ...]], ...]
    fields: Tuple[str, ...]           # message fields in order
    tok_lens: Tuple[int, ...]
    fused_event_dir: bool = False
    price_digits: int = 1             # base-1000 digits after the sign token
    size_mode: str = "single"         # "single" (base-10000) or "digits" (2x base-100)


_TIME = ("time", tuple(range(1000)))
_EVENT = ("event_type", tuple(range(1, 5)))
_SIZE = ("size", tuple(range(10000)))
_SIZE_DIGIT = ("size_digit", tuple(range(100)))
_PRICE = ("price", tuple(range(1000)))
_SIGN = ("sign", (-1, 1))
_DIR = ("direction", (0, 1))
_EVENT_DIR = ("event_dir", tuple(range(8)))

_FIELDS_STD = ("event_type", "direction", "price", "size", "delta_t_s",
               "delta_t_ns", "time_s", "time_ns", "price_ref", "size_ref",
               "time_s_ref", "time_ns_ref")
_FIELDS_23 = ("event_dir",) + _FIELDS_STD[2:]

MODES: Dict[str, ModeSpec] = {
    "22tok": ModeSpec("22tok", (_TIME, _EVENT, _SIZE, _PRICE, _SIGN, _DIR), _FIELDS_STD,
                      (1, 1, 2, 1, 1, 3, 2, 3, 2, 1, 2, 3), False, 1, "single"),
    "23tok": ModeSpec("23tok", (_TIME, _EVENT_DIR, _SIZE_DIGIT, _PRICE, _SIGN), _FIELDS_23,
                      (1, 2, 2, 1, 3, 2, 3, 2, 2, 2, 3), True, 1, "digits"),
    "24tok": ModeSpec("24tok", (_TIME, _EVENT, _SIZE_DIGIT, _PRICE, _SIGN, _DIR), _FIELDS_STD,
                      (1, 1, 2, 2, 1, 3, 2, 3, 2, 2, 2, 3), False, 1, "digits"),
    "26tok": ModeSpec("26tok", (_TIME, _EVENT, _SIZE_DIGIT, _PRICE, _SIGN, _DIR), _FIELDS_STD,
                      (1, 1, 3, 2, 1, 3, 2, 3, 3, 2, 2, 3), False, 2, "digits"),
}


def _is_special(x: np.ndarray) -> np.ndarray:
    return np.isin(x, np.array(SPECIAL_VALS))


def _split_int(x: np.ndarray, n_tokens: int, sign: bool) -> np.ndarray:
    """Base-1000 digits (most significant first); optional sign column first.

    Special values are broadcast to every output column, as the reference's
    ``split_field`` does (``encoding_22tok.py:46-76``).
    """
    x = np.asarray(x, dtype=np.int64)
    a = np.abs(x)
    exps = np.arange(n_tokens - 1, -1, -1)
    digits = (a[..., None] // (1000 ** exps)) % 1000
    cols = [digits]
    if sign:
        s = np.sign(x)
        s = np.where(s == 0, -1, s)
        cols = [s[..., None], digits]
    out = np.concatenate(cols, axis=-1)
    spec = _is_special(x)[..., None]
    return np.where(spec, x[..., None], out)


def _combine(digits: np.ndarray, sign=1) -> np.ndarray:
    """Inverse of ``_split_int`` (``combine_field``): NA if any input is special."""
    digits = np.asarray(digits, dtype=np.int64)
    n = digits.shape[-1]
    exps = np.arange(n - 1, -1, -1)
    val = np.sum(digits * (1000 ** exps), axis=-1) * sign
    spec = _is_special(digits).any(axis=-1) | _is_special(np.asarray(sign))
    return np.where(spec, NA_VAL, val)


class MessageTokenizer:
    """Encoder/decoder for one multi-token mode."""

    def __init__(self, spec: ModeSpec):
        self.spec = spec
        self.vocab = Vocabulary(spec.vocab_fields)
        self.FIELDS = spec.fields
        self.TOK_LENS = np.array(spec.tok_lens)
        self.TOK_DELIM = np.cumsum(self.TOK_LENS[:-1])
        self.MSG_LEN = int(self.TOK_LENS.sum())
        self.FIELD_I = {f: i for i, f in enumerate(self.FIELDS)}
        self.N_REF_FIELDS = 4
        self.N_NEW_FIELDS = len(self.FIELDS) - 4
        self.NEW_MSG_LEN = self.MSG_LEN - int(sum(
            l for f, l in zip(self.FIELDS, self.TOK_LENS) if f.endswith("_ref")))
        starts = np.concatenate([[0], np.cumsum(self.TOK_LENS)])
        self.FIELD_START = {f: int(starts[i]) for i, f in enumerate(self.FIELDS)}
        # absolute-time tokens (time_s, time_ns) of the new message
        self.TIME_START_I = self.FIELD_START["time_s"]
        self.TIME_END_I = self.FIELD_START["time_ns"] + 3 - 1
        self.FIELD_ENC_TYPES = {}
        for f in self.FIELDS:
            base = f[:-4] if f.endswith("_ref") else f
            if base in ("delta_t_s", "delta_t_ns", "time_s", "time_ns"):
                self.FIELD_ENC_TYPES[f] = "time"
            elif base == "size":
                self.FIELD_ENC_TYPES[f] = "size" if spec.size_mode == "single" else "size_digit"
            else:
                self.FIELD_ENC_TYPES[f] = base

    # -- per-position field types (used by the syntax mask) ---------------
    def position_codes(self) -> List[str]:
        """Vocabulary field that each of the MSG_LEN positions draws from."""
        out: List[str] = []
        for f, n in zip(self.FIELDS, self.TOK_LENS):
            base = f[:-4] if f.endswith("_ref") else f
            if base == "price":
                out += ["sign"] + ["price"] * (n - 1)
            else:
                out += [self.FIELD_ENC_TYPES[f]] * n
        return out

    def get_field_from_idx(self, idx):
        idx = np.atleast_1d(np.asarray(idx))
        if np.any(idx > self.MSG_LEN - 1):
            raise ValueError(f"Index ({idx}) must be less than {self.MSG_LEN}")
        fi = np.searchsorted(self.TOK_DELIM, idx, side="right")
        return [self.FIELDS[i] for i in fi]

    # -- encode -------------------------------------------------------------
    def _enc_price(self, x):
        s = _split_int(x, self.spec.price_digits, True)
        sign = self.vocab.codes["sign"].encode(s[..., 0])
        mags = self.vocab.codes["price"].encode(s[..., 1:])
        return np.concatenate([sign[..., None], mags], axis=-1)

    def _enc_size(self, x):
        x = np.asarray(x, dtype=np.int64)
        if self.spec.size_mode == "single":
            return self.vocab.codes["size"].encode(x)[..., None]
        code = self.vocab.codes["size_digit"]
        return np.stack([code.encode(x // 100), code.encode(x % 100)], axis=-1)

    def _enc_time(self, ts, tns, dts=None, dtns=None):
        t_s = _split_int(ts, 2, False)
        t_ns = _split_int(tns, 3, False)
        if dts is None:
            comb = np.concatenate([t_s, t_ns], axis=-1)
        else:
            d_ns = _split_int(dtns, 3, False)
            comb = np.concatenate([np.asarray(dts, np.int64)[..., None], d_ns, t_s, t_ns], axis=-1)
        return self.vocab.codes["time"].encode(comb)

    def encode_msgs(self, msgs: np.ndarray) -> np.ndarray:
        """(n, 14) raw rows -> (n, MSG_LEN) int32 token ids."""
        m = np.asarray(msgs, dtype=np.int64)
        g = lambda name: m[..., RAW_I[name]]
        parts = []
        if self.spec.fused_event_dir:
            ed = (g("event_type") - 1) * 2 + g("direction")
            parts.append(self.vocab.codes["event_dir"].encode(ed)[..., None])
        else:
            parts.append(self.vocab.codes["event_type"].encode(g("event_type"))[..., None])
            parts.append(self.vocab.codes["direction"].encode(g("direction"))[..., None])
        parts.append(self._enc_price(g("price")))
        parts.append(self._enc_size(g("size")))
        parts.append(self._enc_time(g("time_s"), g("time_ns"), g("delta_t_s"), g("delta_t_ns")))
        parts.append(self._enc_price(g("price_ref")))
        parts.append(self._enc_size(g("size_ref")))
        parts.append(self._enc_time(g("time_s_ref"), g("time_ns_ref")))
        out = np.concatenate(parts, axis=-1).astype(np.int32)
        assert out.shape[-1] == self.MSG_LEN
        return out

    # -- decode -------------------------------------------------------------
    def _dec_price(self, toks):
        sign = self.vocab.codes["sign"].decode(toks[..., 0])
        mags = self.vocab.codes["price"].decode(toks[..., 1:])
        return _combine(mags, sign)

    def _dec_size(self, toks):
        if self.spec.size_mode == "single":
            return self.vocab.codes["size"].decode(toks[..., 0])
        code = self.vocab.codes["size_digit"]
        return code.decode(toks[..., 0]) * 100 + code.decode(toks[..., 1])

    def decode_msgs(self, toks: np.ndarray) -> np.ndarray:
        """(n, MSG_LEN) tokens -> (n, 14) raw rows (order id and price_abs NA)."""
        t = np.asarray(toks, dtype=np.int64)
        i = 0
        if self.spec.fused_event_dir:
            ed = self.vocab.codes["event_dir"].decode(t[..., 0])
            et, dr = ed // 2 + 1, ed % 2
            i = 1
        else:
            et = self.vocab.codes["event_type"].decode(t[..., 0])
            dr = self.vocab.codes["direction"].decode(t[..., 1])
            i = 2
        np_ = 1 + self.spec.price_digits
        price = self._dec_price(t[..., i:i + np_]); i += np_
        ns = 1 if self.spec.size_mode == "single" else 2
        size = self._dec_size(t[..., i:i + ns]); i += ns
        tc = self.vocab.codes["time"]
        tm = tc.decode(t[..., i:i + 9]); i += 9
        dts = tm[..., 0]
        dtns = _combine(tm[..., 1:4])
        ts = _combine(tm[..., 4:6])
        tns = _combine(tm[..., 6:9])
        pref = self._dec_price(t[..., i:i + np_]); i += np_
        sref = self._dec_size(t[..., i:i + ns]); i += ns
        tr = tc.decode(t[..., i:i + 5]); i += 5
        tsr = _combine(tr[..., 0:2])
        tnsr = _combine(tr[..., 2:5])
        na = np.full(et.shape, NA_VAL, dtype=np.int64)
        return np.stack([na, et, dr, na, price, size, dts, dtns, ts, tns,
                         pref, sref, tsr, tnsr], axis=-1)


_TOKENIZERS: Dict[str, MessageTokenizer] = {}


def get_tokenizer(mode: str) -> MessageTokenizer:
    if mode not in MODES:
        raise ValueError(f"token_mode {mode!r} is not one of {tuple(MODES)}")
    if mode not in _TOKENIZERS:
        _TOKENIZERS[mode] = MessageTokenizer(MODES[mode])
    return _TOKENIZERS[mode]
