"""The outer LOB model: message encoder + book encoder -> fused trunk -> decoder.

Structure and parameter tree follow the reference's ``PaddedLobPredModel``
(``src/base_model/models/lob_seq_model.py:384-727``):

* ``message_encoder``: ``Embed(vocab, d_model)`` + ``n_message_layers`` layers;
* ``book_encoder``: ``pre_layers_i`` at width ``d_book`` (the mixer is rebuilt
  at that width), ``projection`` Dense(d_book -> d_model), ``post_layers_i``;
* ``fused_s5``: Dense(2*d_model -> d_model) + ``n_fused_layers`` layers (hybrid
  attention positions live here only);
* ``decoder``: Dense(d_model -> vocab); the head is a log-softmax.

The book input is one row per message; ``forward`` repeats each row over the
message's tokens on the device, as the reference's ``repeat_book`` does.  The
training entry point returns the mean next-token cross-entropy; the logits
never materialise in float32 on the CUDA path (fused CE kernel).
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .common import Dense
from .layers import SequenceLayer, StackedEncoder


class LobBookEncoder(nn.Module):
    def __init__(self, factory_at: Callable[[int], nn.Module], d_book: int, d_model: int,
                 n_pre: int, n_post: int, activation: str, prenorm: bool, dropout: float):
        super().__init__()
        self.n_pre, self.n_post = n_pre, n_post
        for i in range(n_pre):
            self.add_module(f"pre_layers_{i}", SequenceLayer(factory_at(d_book), d_book, activation, prenorm, dropout))
        self.projection = Dense(d_book, d_model)
        self.compute_dtype = torch.float32
        for i in range(n_post):
            self.add_module(f"post_layers_{i}", SequenceLayer(factory_at(d_model), d_model, activation, prenorm, dropout))

    @property
    def pre_layers(self):
        return [getattr(self, f"pre_layers_{i}") for i in range(self.n_pre)]

    @property
    def post_layers(self):
        return [getattr(self, f"post_layers_{i}") for i in range(self.n_post)]

    def forward(self, x):
        for l in self.pre_layers:
            x = l(x)
        x = self._project(x)
        for l in self.post_layers:
            x = l(x)
        return x

    def _project(self, x):
        """The d_book -> d_model projection: bf16 (K padded to 8) on CUDA, else fp32."""
        if x.is_cuda and self.compute_dtype == torch.bfloat16:
            from ..ops.linear import linear_bf16
            return linear_bf16(x, self.projection.kernel, self.projection.bias)
        return self.projection(x)

    def initial_state(self, batch, device=None):
        return ([l.initial_state(batch, device) for l in self.pre_layers],
                [l.initial_state(batch, device) for l in self.post_layers])

    @torch.no_grad()
    def prefill(self, x, max_cache_len=None):
        pre, post = [], []
        for l in self.pre_layers:
            st, x = l.prefill(x, max_cache_len)
            pre.append(st)
        x = self._project(x)
        for l in self.post_layers:
            st, x = l.prefill(x, max_cache_len)
            post.append(st)
        return (pre, post), x

    def step(self, states, x):
        pre, post = states
        npre, npost = [], []
        for s, l in zip(pre, self.pre_layers):
            s, x = l.step(s, x)
            npre.append(s)
        x = self.projection(x)
        for s, l in zip(post, self.post_layers):
            s, x = l.step(s, x)
            npost.append(s)
        return (npre, npost), x


class LobModel(nn.Module):
    def __init__(self, factory_at: Callable[[int], nn.Module], vocab_size: int, d_model: int,
                 d_book: int = 503, n_message_layers: int = 2, n_fused_layers: int = 6,
                 n_book_pre_layers: int = 1, n_book_post_layers: int = 1,
                 activation: str = "half_glu1", prenorm: bool = True, dropout: float = 0.0,
                 msg_len: int = 22, use_book_data: bool = True,
                 attn_factory_at: Optional[Callable[[int], nn.Module]] = None,
                 attn_layers: Sequence[int] = ()):
        super().__init__()
        self.vocab_size, self.d_model, self.d_book, self.msg_len = vocab_size, d_model, d_book, msg_len
        self.use_book_data = use_book_data
        self.message_encoder = StackedEncoder(lambda: factory_at(d_model), d_model, n_message_layers,
                                              use_embed_layer=True, vocab_size=vocab_size,
                                              activation=activation, prenorm=prenorm, dropout=dropout)
        if use_book_data:
            self.book_encoder = LobBookEncoder(factory_at, d_book, d_model, n_book_pre_layers,
                                               n_book_post_layers, activation, prenorm, dropout)
        attn_factory = (lambda: attn_factory_at(d_model)) if attn_factory_at is not None else None
        self.fused_s5 = StackedEncoder(lambda: factory_at(d_model), d_model, n_fused_layers,
                                       d_input=(2 if use_book_data else 1) * d_model,
                                       activation=activation, prenorm=prenorm, dropout=dropout,
                                       attn_factory=attn_factory, attn_layers=attn_layers)
        self.decoder = Dense(d_model, vocab_size)

    # -- helpers -----------------------------------------------------------------------
    def repeat_book(self, book: torch.Tensor, n_tokens: int) -> torch.Tensor:
        """(B, n_msgs, d_book) per-message rows -> (B, n_tokens, d_book)."""
        if book.shape[1] == n_tokens:
            return book
        rep = n_tokens // book.shape[1]
        return book.repeat_interleave(rep, dim=1)

    def hidden(self, tokens: torch.Tensor, book: Optional[torch.Tensor]) -> torch.Tensor:
        xm = self.message_encoder(tokens)
        if self.use_book_data:
            xb = self.book_encoder(self.repeat_book(book, tokens.shape[1]))
            x = torch.cat([xm, xb.to(xm.dtype)], dim=-1)
        else:
            x = xm
        return self.fused_s5(x)

    def forward(self, tokens, book=None):
        """Log-probabilities (B, L, vocab) in float32 (the reference's ``__call_ar__``)."""
        h = self.hidden(tokens, book)
        return F.log_softmax(self.decoder(h).float(), dim=-1)

    def loss(self, tokens, book, labels, ignore_times: bool = False, tokenizer=None):
        """Mean next-token cross-entropy and per-position CE (batch mean), like
        ``_compute_ce_unified`` (``training/train_helpers.py:755-783``).  With
        ``ignore_times`` the absolute-time tokens of every message are dropped."""
        h = self.hidden(tokens, book)
        B, L = labels.shape
        # the kept positions are known on the host: no device round trip in the step
        keep = torch.ones(L, dtype=torch.bool)
        if ignore_times:
            pos = torch.arange(L) % self.msg_len
            keep = (pos < tokenizer.TIME_START_I) | (pos > tokenizer.TIME_END_I)
        n_keep = int(keep.sum())
        idx = None if n_keep == L else keep.nonzero()[:, 0].to(labels.device, non_blocking=True)
        if h.is_cuda:
            from ..ops.cross_entropy import linear_cross_entropy_mean
            w = keep.to(labels.device, non_blocking=True).float().expand(B, L) / (B * n_keep)
            loss, ce = linear_cross_entropy_mean(h, self.decoder.kernel, self.decoder.bias, labels, w)
        else:
            logits = self.decoder(h).float()
            ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1),
                                 reduction="none").reshape(labels.shape)
            loss = (ce if idx is None else ce.index_select(1, idx)).mean()
        ce_pos = (ce if idx is None else ce.index_select(1, idx)).mean(0)
        return loss, ce_pos

    # -- decode ------------------------------------------------------------------------
    def initial_state(self, batch, device=None):
        return (self.message_encoder.initial_state(batch, device),
                self.book_encoder.initial_state(batch, device) if self.use_book_data else None,
                self.fused_s5.initial_state(batch, device))

    @torch.no_grad()
    def prefill(self, tokens, book=None, max_cache_len=None):
        """Forward over a context that returns (decode state, log-probs of the last token)."""
        sm, xm = self.message_encoder.prefill(tokens, max_cache_len)
        sb = None
        if self.use_book_data:
            sb, xb = self.book_encoder.prefill(self.repeat_book(book, tokens.shape[1]), max_cache_len)
            x = torch.cat([xm, xb.to(xm.dtype)], dim=-1)
        else:
            x = xm
        sf, h = self.fused_s5.prefill(x, max_cache_len)
        return (sm, sb, sf), F.log_softmax(self.decoder(h[:, -1:]).float(), dim=-1)

    def step(self, state, tokens, book=None):
        """Recurrent step over ``tokens`` (B, l) with book rows (B, l, d_book) -> (state, logp)."""
        state, h = self.step_hidden(state, tokens, book)
        return state, F.log_softmax(self.decoder(h).float(), dim=-1)

    def step_hidden(self, state, tokens, book=None):
        """``step`` without the decoder: (state, last hidden (B, l, d_model))."""
        sm, sb, sf = state
        sm, xm = self.message_encoder.step(sm, tokens)
        if self.use_book_data:
            sb, xb = self.book_encoder.step(sb, book)
            x = torch.cat([xm, xb.to(xm.dtype)], dim=-1)
        else:
            x = xm
        sf, h = self.fused_s5.step(sf, x)
        return (sm, sb, sf), h
