"""Message-level perplexity: a loss that does not depend on the tokenizer.

Per-token cross-entropy changes with the encoding (22/23/24/26 tokens per
message); the negative log-likelihood of a whole message does not: by the
chain rule it is the sum of its tokens' NLLs, and the encodings are lossless
bijections.  Following the reference's definition
(``src/base_model/evaluation/message_perplexity.py``):

* ``full``  -- every token of the message;
* ``main``  -- the message's own content: event type, direction, price, size
  and the inter-arrival time (the absolute time is a deterministic function
  of the past plus the delta, and the reference fields point at an earlier
  order), so ``full = main + absolute_time + reference`` exactly.

Reported per variant: nats per message, bits per message and perplexity
(the exponential), plus the per-field nats.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np
import torch
import torch.nn.functional as F

MAIN_FIELDS = ("event_type", "event_dir", "direction", "price", "size", "delta_t_s", "delta_t_ns")
TIME_FIELDS = ("time_s", "time_ns")


def field_role(name: str) -> str:
    if name.endswith("_ref"):
        return "reference"
    if name in TIME_FIELDS:
        return "absolute_time"
    if name in MAIN_FIELDS:
        return "main"
    raise ValueError(f"unknown message field {name!r}")


@dataclass
class MessagePerplexity:
    n_messages: int
    per_field_nats: Dict[str, float]          # mean nats per message, per field
    roles: Dict[str, float] = field(default_factory=dict)

    @property
    def main_nats(self) -> float:
        return self.roles["main"]

    @property
    def full_nats(self) -> float:
        return sum(self.roles.values())

    def as_dict(self) -> Dict:
        def view(n):
            return {"nats_per_message": n, "bits_per_message": n / math.log(2),
                    "perplexity": math.exp(min(n, 700.0))}
        return {"n_messages": self.n_messages, "main": view(self.main_nats), "full": view(self.full_nats),
                "roles": dict(self.roles), "per_field_nats": dict(self.per_field_nats)}


def token_nll(model, tokens: torch.Tensor, labels: torch.Tensor, book: Optional[torch.Tensor]) -> torch.Tensor:
    """(B, L) per-token NLL in nats (float32)."""
    with torch.no_grad():
        logp = model(tokens, book)
        return -logp.gather(-1, labels.unsqueeze(-1)).squeeze(-1).float()


def message_perplexity_from_nll(nll: torch.Tensor, tokenizer) -> MessagePerplexity:
    """nll (B, L) with L a multiple of MSG_LEN, aligned with the label sequence."""
    L = tokenizer.MSG_LEN
    B, T = nll.shape
    per_msg = nll.reshape(B, T // L, L).double()
    n = B * (T // L)
    starts = np.concatenate([[0], np.cumsum(tokenizer.TOK_LENS)])
    per_field = {}
    roles: Dict[str, float] = {"main": 0.0, "absolute_time": 0.0, "reference": 0.0}
    for i, f in enumerate(tokenizer.FIELDS):
        v = float(per_msg[..., starts[i]:starts[i + 1]].sum(-1).mean())
        per_field[f] = v
        roles[field_role(f)] += v
    return MessagePerplexity(n, per_field, roles)


def message_perplexity(model, batches, tokenizer) -> MessagePerplexity:
    """Average over an iterable of (tokens, labels, book) batches."""
    acc, total = None, 0
    for tokens, labels, book in batches:
        dev = next(model.parameters()).device
        nll = token_nll(model, tokens.to(dev), labels.to(dev), book.to(dev) if book is not None else None)
        mp = message_perplexity_from_nll(nll.cpu(), tokenizer)
        w = mp.n_messages
        if acc is None:
            acc = {k: v * w for k, v in mp.per_field_nats.items()}
        else:
            for k, v in mp.per_field_nats.items():
                acc[k] += v * w
        total += w
    per_field = {k: v / total for k, v in acc.items()}
    roles = {"main": 0.0, "absolute_time": 0.0, "reference": 0.0}
    for f, v in per_field.items():
        roles[field_role(f)] += v
    return MessagePerplexity(total, per_field, roles)
