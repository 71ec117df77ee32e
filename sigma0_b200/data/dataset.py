"""Windowed next-token dataset over message/book arrays.

A sample is a window of ``n_messages`` consecutive messages.  Messages are
encoded with the active tokenizer and flattened; the input is the token stream
shifted right by one with a START token in front, the label is the unshifted
stream (the reference's ``no_mask``, ``src/base_model/data/lobster_dataloader.py:657-668``).
The book input is one row per message (the state before that message) after
the volume-image transform; the model repeats it to token resolution on the
device (the reference's ``repeat_book``, ``training/train_helpers.py:1383``).

Other objectives (``mask=``): ``"inference"``, ``"random"``, ``"causal"`` or any
``fn(seq (n_messages, MSG_LEN), rng) -> (masked seq, label)`` from ``data/masks.py``;
these return the flattened masked window and a scalar label.  ``book_ablation`` replaces
the book input by zeros, noise or a shuffled copy (seeded per window).

Sources are either in-memory :class:`~sigma0_b200.data.synthetic.SyntheticDay`
objects or ``.npy`` message/book file pairs (the reference's on-disk layout;
``.npy.zst`` files are decompressed with the ``zstandard`` module or the system libzstd).
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence

import numpy as np
import torch

from ..encoding import get_tokenizer, START_TOK
from . import masks as M
from .book_transform import transform_books_numpy


class LobWindowDataset(torch.utils.data.Dataset):
    def __init__(self, msgs: Sequence[np.ndarray], books: Sequence[np.ndarray], n_messages: int,
                 token_mode: str = "22tok", book_depth: int = 500, use_book_data: bool = True,
                 stride: Optional[int] = None, return_raw_msgs: bool = False, mask="no_mask",
                 book_ablation: str = "real", seed: int = 0, random_offsets: bool = False):
        from ..encoding.tok1 import encoding_mode
        self.one_token = token_mode == "1tok"      # 24tok messages as one row of 24 field ids each
        self.tok = get_tokenizer(encoding_mode(token_mode))
        if self.one_token and mask == "no_mask":
            mask = "no_mask_1tok"
        self.mask, self.book_ablation, self.seed = mask, book_ablation, seed
        # random_offsets: every epoch shifts each day's windows by a seeded offset in
        # [0, n_messages) (the reference's random_offsets_train), clipped to the day's end
        self.random_offsets, self.epoch = random_offsets, 0
        self.n = n_messages
        self.book_depth = book_depth
        self.use_book = use_book_data
        self.return_raw = return_raw_msgs
        self.msgs = list(msgs)
        self.books = list(books)
        stride = stride or n_messages
        self.index = []
        for f, m in enumerate(self.msgs):
            for s in range(0, m.shape[0] - n_messages + 1, stride):
                self.index.append((f, s))

    @classmethod
    def from_days(cls, days, n_messages, **kw):
        return cls([d.msgs for d in days], [d.books for d in days], n_messages, **kw)

    @classmethod
    def from_dir(cls, directory: str, n_messages: int, **kw):
        def names(tag):
            fs = {f[:-4] if f.endswith(".zst") else f for f in os.listdir(directory)
                  if f.endswith(tag + ".npy") or f.endswith(tag + ".npy.zst")}
            return sorted(fs)
        msgs = [M.load_npy(os.path.join(directory, f)) for f in names("message")]
        books = [M.load_npy(os.path.join(directory, f)) for f in names("book")]
        return cls(msgs, books, n_messages, **kw)

    def __len__(self):
        return len(self.index)

    def set_epoch(self, epoch: int) -> None:
        self.epoch = int(epoch)

    def __getitem__(self, i):
        f, s = self.index[i]
        if self.random_offsets:
            off = int(np.random.default_rng([self.seed, self.epoch, f]).integers(0, self.n))
            s = min(s + off, self.msgs[f].shape[0] - self.n)
        raw = np.asarray(self.msgs[f][s:s + self.n])
        enc = self.tok.encode_msgs(raw)
        if self.mask == "no_mask":
            x = enc.reshape(-1)
            y = x.copy()
            x = np.concatenate([[START_TOK], x[:-1]])
        elif self.mask == "no_mask_1tok":      # per-field local indices, shifted by one message
            from ..encoding.tok1 import global_to_local
            (x, _), y = M.no_mask_1tok(enc)
            x, y = global_to_local(x), global_to_local(y)
        elif self.mask == "inference":
            (x, _), y = M.inference_mask(enc)
        else:
            rng = np.random.default_rng([self.seed, f, s])
            if self.mask == "random":
                m, y = M.random_mask(self.tok, enc, rng)
            elif self.mask == "causal":
                m, y = M.causal_mask(self.tok, enc, rng)
            else:
                m, y = self.mask(enc, rng)
            x = np.asarray(m).reshape(-1)
        out = [torch.from_numpy(np.asarray(x, dtype=np.int64)), torch.from_numpy(np.asarray(y, dtype=np.int64))]
        if self.use_book:
            b = transform_books_numpy(np.asarray(self.books[f][s:s + self.n]), self.book_depth)
            b = M.ablate_books(b, self.book_ablation, (f, s))
            out.append(torch.from_numpy(np.ascontiguousarray(b)))
        if self.return_raw:
            out.append(torch.from_numpy(raw))
        return tuple(out)


def collate(batch):
    return tuple(torch.stack(z) for z in zip(*batch))
