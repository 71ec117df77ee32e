"""Windowed next-token dataset over message/book arrays.

A sample is a window of ``n_messages`` consecutive messages.  Messages are
encoded with the active tokenizer and flattened; the input is the token stream
shifted right by one with a START token in front, the label is the unshifted
stream (the reference's ``no_mask``, ``src/base_model/data/lobster_dataloader.py:657-668``).
The book input is one row per message (the state before that message) after
the volume-image transform; the model repeats it to token resolution on the
device (the reference's ``repeat_book``, ``training/train_helpers.py:1383``).

Sources are either in-memory :class:`~sigma0_b200.data.synthetic.SyntheticDay`
objects or ``.npy`` message/book file pairs (the reference's on-disk layout,
optionally zstd-compressed ``.npy.zst`` is not supported without zstandard).
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence

import numpy as np
import torch

from ..encoding import get_tokenizer, START_TOK
from .book_transform import transform_books_numpy


class LobWindowDataset(torch.utils.data.Dataset):
    def __init__(self, msgs: Sequence[np.ndarray], books: Sequence[np.ndarray], n_messages: int,
                 token_mode: str = "22tok", book_depth: int = 500, use_book_data: bool = True,
                 stride: Optional[int] = None, return_raw_msgs: bool = False):
        self.tok = get_tokenizer(token_mode)
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
        mf = sorted(f for f in os.listdir(directory) if f.endswith("message.npy"))
        bf = sorted(f for f in os.listdir(directory) if f.endswith("book.npy"))
        msgs = [np.load(os.path.join(directory, f), mmap_mode="r") for f in mf]
        books = [np.load(os.path.join(directory, f), mmap_mode="r") for f in bf]
        return cls(msgs, books, n_messages, **kw)

    def __len__(self):
        return len(self.index)

    def __getitem__(self, i):
        f, s = self.index[i]
        raw = np.asarray(self.msgs[f][s:s + self.n])
        x = self.tok.encode_msgs(raw).reshape(-1)
        y = x.copy()
        x = np.concatenate([[START_TOK], x[:-1]]).astype(np.int64)
        out = [torch.from_numpy(x), torch.from_numpy(y.astype(np.int64))]
        if self.use_book:
            b = transform_books_numpy(np.asarray(self.books[f][s:s + self.n]), self.book_depth)
            out.append(torch.from_numpy(b))
        if self.return_raw:
            out.append(torch.from_numpy(raw))
        return tuple(out)


def collate(batch):
    return tuple(torch.stack(z) for z in zip(*batch))
