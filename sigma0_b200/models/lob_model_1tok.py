"""The 1-token-per-message LOB model: one sequence position per message.

Structure and parameter tree follow the reference's ``OneTokenPaddedLobPredModel``
(``src/base_model/models/lob_seq_model.py:1071-1230``):

* ``field_embedding``: the sum of 24 per-field embeddings ``field_i`` of
  ``(V_i + 4, d_model)`` over the 24 fields of a message (local field indices,
  ``encoding/tok1.py``) -- one CUDA kernel (``csrc/embed.cu``) on the GPU;
* ``book_encoder`` and ``fused_s5``: as in the token-level model (the book row of a
  message meets the message embedding directly, no repetition);
* ``decoder``: 24 classification heads ``head_i`` (Dense d_model -> V_i + 4), each a
  log-softmax over its field's local vocabulary.  The heads run as one GEMM over the
  concatenated kernels; the per-field softmax is taken on slices of its output.

The loss is the reference's field-head cross-entropy (``training/train_helpers.py:755-770``):
the per-field CE of every (message, field), with the absolute-time fields dropped under
``ignore_times``, averaged.  There is no message encoder (the embedding is the message
representation).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..encoding import tok1
from .common import Dense, Embed, embed_sum
from .layers import StackedEncoder
from .lob_model import LobBookEncoder


class FieldEmbedding(nn.Module):
    def __init__(self, field_vocab_sizes: Sequence[int], d_model: int):
        super().__init__()
        self.n = len(field_vocab_sizes)
        for i, v in enumerate(field_vocab_sizes):
            self.add_module(f"field_{i}", Embed(int(v), d_model))

    def tables(self) -> List[torch.Tensor]:
        return [getattr(self, f"field_{i}").embedding for i in range(self.n)]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x (..., n_fields) local indices -> (..., d_model)."""
        return embed_sum(x, self.tables())


class MultiFieldDecoder(nn.Module):
    def __init__(self, d_model: int, field_vocab_sizes: Sequence[int]):
        super().__init__()
        self.sizes = [int(v) for v in field_vocab_sizes]
        for i, v in enumerate(self.sizes):
            self.add_module(f"head_{i}", Dense(d_model, v))

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """All heads as one GEMM: (..., sum of field vocabularies) in float32."""
        heads = [getattr(self, f"head_{i}") for i in range(len(self.sizes))]
        w = torch.cat([hd.kernel for hd in heads], 1)
        b = torch.cat([hd.bias for hd in heads], 0)
        if h.is_cuda and h.dtype == torch.bfloat16:
            return (h @ w.to(torch.bfloat16)).float() + b
        return h.float() @ w + b

    def forward(self, h: torch.Tensor) -> List[torch.Tensor]:
        """The 24 per-field log-probabilities (float32)."""
        return [F.log_softmax(z, -1) for z in torch.split(self.logits(h), self.sizes, -1)]


class OneTokenLobModel(nn.Module):
    def __init__(self, factory_at: Callable[[int], nn.Module], d_model: int, d_book: int = 503,
                 n_fused_layers: int = 6, n_book_pre_layers: int = 1, n_book_post_layers: int = 1,
                 activation: str = "half_glu1", prenorm: bool = True, dropout: float = 0.0,
                 use_book_data: bool = True, field_vocab_sizes: Sequence[int] = tok1.FIELD_VOCAB_SIZES_WITH_SPECIAL,
                 attn_factory_at: Optional[Callable[[int], nn.Module]] = None, attn_layers: Sequence[int] = ()):
        super().__init__()
        self.d_model, self.d_book, self.use_book_data = d_model, d_book, use_book_data
        self.msg_len = 1
        self.n_fields = len(field_vocab_sizes)
        self.field_embedding = FieldEmbedding(field_vocab_sizes, d_model)
        if use_book_data:
            self.book_encoder = LobBookEncoder(factory_at, d_book, d_model, n_book_pre_layers, n_book_post_layers,
                                               activation, prenorm, dropout)
        attn_factory = (lambda: attn_factory_at(d_model)) if attn_factory_at is not None else None
        self.fused_s5 = StackedEncoder(lambda: factory_at(d_model), d_model, n_fused_layers,
                                       d_input=(2 if use_book_data else 1) * d_model, activation=activation,
                                       prenorm=prenorm, dropout=dropout, attn_factory=attn_factory,
                                       attn_layers=attn_layers)
        self.decoder = MultiFieldDecoder(d_model, field_vocab_sizes)

    def hidden(self, x_m: torch.Tensor, book: Optional[torch.Tensor]) -> torch.Tensor:
        xm = self.field_embedding(x_m)
        if self.use_book_data:
            xb = self.book_encoder(book)
            x = torch.cat([xm.to(xb.dtype), xb], dim=-1)
        else:
            x = xm
        return self.fused_s5(x)

    def forward(self, x_m, book=None) -> List[torch.Tensor]:
        """Per-field log-probabilities, each (B, L, V_i + 4) -- the reference's ``__call_training__``."""
        return self.decoder(self.hidden(x_m, book))

    def loss(self, x_m, book, labels, ignore_times: bool = False, tokenizer=None):
        """Mean field-head cross-entropy; ``labels`` (B, L, 24) local indices.  Returns the
        loss and the per-field CE (mean over batch and messages)."""
        logp = self.forward(x_m, book)
        fields = range(self.n_fields)
        if ignore_times and tokenizer is not None:
            fields = [i for i in fields if not (tokenizer.TIME_START_I <= i <= tokenizer.TIME_END_I)]
        ce = torch.stack([F.nll_loss(logp[i].reshape(-1, logp[i].shape[-1]), labels[..., i].reshape(-1),
                                     reduction="none").reshape(labels.shape[:-1]) for i in fields], -1)
        return ce.mean(), ce.mean(dim=(0, 1))

    # -- decode ------------------------------------------------------------------------
    def initial_state(self, batch, device=None):
        return (self.book_encoder.initial_state(batch, device) if self.use_book_data else None,
                self.fused_s5.initial_state(batch, device))

    @torch.no_grad()
    def prefill(self, x_m, book=None, max_cache_len=None):
        xm = self.field_embedding(x_m)
        sb = None
        if self.use_book_data:
            sb, xb = self.book_encoder.prefill(book, max_cache_len)
            x = torch.cat([xm.to(xb.dtype), xb], dim=-1)
        else:
            x = xm
        sf, h = self.fused_s5.prefill(x, max_cache_len)
        return (sb, sf), self.decoder(h[:, -1:])

    def step(self, state, x_m, book=None):
        """One or more messages (B, l, 24) through the recurrence -> (state, per-field logp)."""
        sb, sf = state
        xm = self.field_embedding(x_m)
        if self.use_book_data:
            sb, xb = self.book_encoder.step(sb, book)
            x = torch.cat([xm.to(xb.dtype), xb], dim=-1)
        else:
            x = xm
        sf, h = self.fused_s5.step(sf, x)
        return (sb, sf), self.decoder(h)
