"""Syntax masks and sampling for token-by-token message generation.

``syntax_validation_matrix`` is the (MSG_LEN, vocab) boolean table of tokens
allowed at each message position, built like the reference's
(``src/base_model/inference/validation.py:56-97``): each position allows the
tokens of its field's vocabulary; sign positions allow both signs; MASK and
HIDDEN are never generated; START is blocked (the ``legacy_recurrent`` mode
of the reference re-allows it); NA is allowed only in the reference fields.

``sample`` implements ``fill_predicted_tok`` (``:217``): argmax for
``top_n == 1``, sampling among the ``top_n`` most likely tokens for
``top_n > 1``, and the full distribution for ``top_n == -1``.
"""
from __future__ import annotations

import numpy as np
import torch

from ..encoding.tokenizer import MASK_TOK, HIDDEN_TOK, NA_TOK, START_TOK, MessageTokenizer


def syntax_validation_matrix(tok: MessageTokenizer, block_start_tok: bool = True, vocab_size=None) -> np.ndarray:
    V = vocab_size or len(tok.vocab)
    mask = np.zeros((tok.MSG_LEN, V), dtype=bool)
    for i, field in enumerate(tok.position_codes()):
        code = tok.vocab.codes[field]
        mask[i, code.toks] = True
    mask[:, MASK_TOK] = False
    mask[:, HIDDEN_TOK] = False
    if block_start_tok:
        mask[:, START_TOK] = False
    mask[:, NA_TOK] = False
    mask[tok.NEW_MSG_LEN:, NA_TOK] = True
    return mask


def sample(logits: torch.Tensor, top_n: int = 1, generator=None) -> torch.Tensor:
    """logits (B, V) (already masked with -inf) -> token ids (B,)."""
    if top_n == 1:
        return logits.argmax(-1)
    if top_n > 1:
        vals, idx = logits.topk(top_n, dim=-1)
        p = torch.softmax(vals.float(), -1)
        pick = torch.multinomial(p, 1, generator=generator)
        return idx.gather(-1, pick)[:, 0]
    p = torch.softmax(logits.float(), -1)
    return torch.multinomial(p, 1, generator=generator)[:, 0]
