"""1-token-per-message field layout over the 24-token encoding.

Each of the 24 positions of a 24tok message gets its own local index space
(4 specials + that field's real values), so a model can use one embedding and
one classification head per field.  Global ids come from the 24tok vocabulary
(``src/base_model/encoding/encoding_1tok.py:22-136``).
"""
from __future__ import annotations

import numpy as np

from .tokenizer import N_SPECIAL, get_tokenizer

_T24 = get_tokenizer("24tok")
FIELD_TYPES = tuple(_T24.position_codes())
N_FIELDS = len(FIELD_TYPES)  # 24
N_SPECIAL_TOKENS = N_SPECIAL
FIELD_VOCAB_SIZES = tuple(len(_T24.vocab.codes[f].values) for f in FIELD_TYPES)
FIELD_VOCAB_SIZES_WITH_SPECIAL = tuple(v + N_SPECIAL for v in FIELD_VOCAB_SIZES)
FIELD_OFFSETS = np.array([_T24.vocab.codes[f].offset for f in FIELD_TYPES], dtype=np.int32)
FIELD_NAMES = (
    "event_type", "direction", "price_sign", "price_mag", "size_high", "size_low",
    "delta_t_s", "delta_t_ns_0", "delta_t_ns_1", "delta_t_ns_2",
    "time_s_0", "time_s_1", "time_ns_0", "time_ns_1", "time_ns_2",
    "price_ref_sign", "price_ref_mag", "size_ref_high", "size_ref_low",
    "time_s_ref_0", "time_s_ref_1", "time_ns_ref_0", "time_ns_ref_1", "time_ns_ref_2",
)


def global_to_local(tokens) -> np.ndarray:
    t = np.asarray(tokens)
    return np.where(t < N_SPECIAL, t, t - FIELD_OFFSETS + N_SPECIAL).astype(np.int32)


def local_to_global(tokens) -> np.ndarray:
    t = np.asarray(tokens)
    return np.where(t < N_SPECIAL, t, t + FIELD_OFFSETS - N_SPECIAL).astype(np.int32)


def encoding_mode(token_mode: str) -> str:
    """The message encoding under a run's ``token_mode``: the 1-token model reads 24tok
    messages (and maps them to per-field local indices); other modes are themselves."""
    return "24tok" if token_mode == "1tok" else token_mode
