"""Batched order books: one warp per book on the GPU, the CPU oracle otherwise.

``BatchedEngine`` holds every book's sides and trade rows as device tensors
``(n_books, n_orders, 6)`` / ``(n_books, n_trades, 8)`` (int32) and applies a
message per book (or a whole stream per book) in one kernel launch
(``csrc/engine.cu``).  On CPU, or for cancel modes 2/3 (random fallback), it
drives one :class:`~sigma0_b200.engine.book.OrderBook` per book.
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .book import EngineConfig, OrderBook, init_msgs_from_l2


class BatchedEngine:
    def __init__(self, n_books: int, cfg: EngineConfig = EngineConfig(), device="cpu"):
        self.n, self.cfg = n_books, cfg
        self.device = torch.device(device)
        self.on_gpu = self.device.type == "cuda" and cfg.cancel_mode <= 1
        self.reset()

    def reset(self):
        c = self.cfg
        if self.on_gpu:
            self.asks = torch.full((self.n, c.n_orders, 6), -1, dtype=torch.int32, device=self.device)
            self.bids = torch.full_like(self.asks, -1)
            self.trades = torch.full((self.n, c.n_trades, 8), -1, dtype=torch.int32, device=self.device)
        else:
            self.books: List[OrderBook] = [OrderBook(c, seed=c.seed + i) for i in range(self.n)]

    def reset_from_l2(self, l2: torch.Tensor, time=(34200, 0)):
        """l2 (n_books, 4*levels) snapshots -> fresh books (``OrderBook.reset``)."""
        self.reset()
        l2n = l2.cpu().numpy() if isinstance(l2, torch.Tensor) else np.asarray(l2)
        msgs = np.stack([init_msgs_from_l2(r, self.cfg, time) for r in l2n])
        self.process(msgs)

    def process(self, msgs):
        """msgs (n_books, 8) or (n_books, M, 8) engine rows, applied in order per book."""
        if isinstance(msgs, np.ndarray):
            msgs = torch.from_numpy(msgs)
        if msgs.dim() == 2:
            msgs = msgs[:, None]
        if self.on_gpu:
            from ..ops._ext import ext
            m = msgs.to(device=self.device, dtype=torch.int32).contiguous()
            c = self.cfg
            ext().eng_process(self.asks, self.bids, self.trades, m, c.init_id, c.book_depth, c.cancel_mode,
                              c.type_4_interpretation, c.check_book_fill)
            return
        mm = msgs.cpu().numpy()
        for b, ob in enumerate(self.books):
            for row in mm[b]:
                ob.process(row)

    def l2(self, levels: Optional[int] = None) -> torch.Tensor:
        levels = levels or self.cfg.book_depth
        if self.on_gpu:
            from ..ops._ext import ext
            return ext().eng_l2(self.asks, self.bids, levels)
        return torch.from_numpy(np.stack([ob.l2(levels) for ob in self.books]).astype(np.int64))

    def sides(self):
        """(asks, bids) as int64 numpy arrays (for tests and lookups)."""
        if self.on_gpu:
            return self.asks.cpu().numpy().astype(np.int64), self.bids.cpu().numpy().astype(np.int64)
        return (np.stack([ob.asks for ob in self.books]), np.stack([ob.bids for ob in self.books]))

    def trade_rows(self):
        if self.on_gpu:
            return self.trades.cpu().numpy().astype(np.int64)
        return np.stack([ob.trades for ob in self.books])
