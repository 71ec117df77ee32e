"""Autoregressive order-flow generation with the matching engine in the loop.

Per message and per book (``_generate_msg``,
``src/base_model/inference/generate.py:870-1061``):

1. tokens up to the last delta-t token are sampled one model step at a time
   under the position's syntax mask;
2. the absolute-time tokens are computed from the previous time plus the
   sampled delta-t (``_add_time_tokens`` ``:759``) and rolled through the model;
3. the remaining (reference) tokens are sampled;
4. the message is decoded, its order id resolved (new orders get the running
   counter, cancels look up the referenced order by exact timestamp, then by
   closest time at the price: ``get_sim_msg`` ``:386``), and applied to the
   book; the new mid, L2 state and the next book image follow
   (``_get_new_mid_price`` ``:703``, ``transform_L2_state``).

On the GPU all of a message is device work: recurrent decode kernels per
layer (``m3_decode_step``), a fused masked sampler reading the decoder's fp32
logits (``gen_sample``), a time-token kernel, and one warp-per-book kernel
doing steps 4 (``gen_apply``).  With ``use_graphs`` the whole message
(MSG_LEN model steps + engine) is captured once as a CUDA graph and replayed,
which removes the per-kernel launch cost of ~MSG_LEN x layers x 8 launches.

On the CPU the same loop runs through the torch recurrences and the numpy
``OrderBook`` (this path is also the oracle for the GPU kernels).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from ..encoding.tokenizer import NA_VAL, MessageTokenizer, get_tokenizer
from ..engine.book import EngineConfig, OrderBook, book_from_l2
from ..data.book_transform import transform_l2_numpy
from .validation import syntax_validation_matrix

NEG_RET = -999_999_999


# ---------------------------------------------------------------------------
# layout of the message tokens for the device kernels
# ---------------------------------------------------------------------------

def gen_layout(tok: MessageTokenizer, tick: int, img_levels: int, l2_levels: int) -> List[int]:
    """The 22 ints of the device ``GenLayout`` struct for tokenizer ``tok``."""
    v = tok.vocab.codes
    fs = tok.FIELD_START
    fused = tok.spec.fused_event_dir
    ev_pos = 0
    ev_off = v["event_dir"].offset if fused else v["event_type"].offset
    dir_pos = 0 if fused else fs["direction"]
    dir_off = 0 if fused else v["direction"].offset
    size_digits = 0 if tok.spec.size_mode == "single" else 1
    size_code = v["size"] if size_digits == 0 else v["size_digit"]
    return [tok.MSG_LEN, int(fused), ev_pos, ev_off, dir_pos, dir_off,
            v["sign"].offset, v["price"].offset, tok.spec.price_digits, fs["price"], fs["price_ref"],
            size_digits, size_code.offset, len(size_code.values), fs["size"], fs["size_ref"],
            v["time"].offset, fs["delta_t_s"], fs["time_s_ref"],
            tick, img_levels, l2_levels]


def safe_mid_price(best_ask: int, best_bid: int, tick: int) -> int:
    """``_get_safe_mid_price`` (``generate.py:674``): one-sided books quote a tick away."""
    a, b = int(best_ask), int(best_bid)
    case = (a <= 0) * 1 + (b <= 0) * 2
    p = [(a + b) // 2, b + tick, a - tick, 0][case]
    return (p // tick) * tick


def _best_quotes(ob: OrderBook):
    asks = ob.asks[:, 0]
    live = asks[asks != -1]
    ba = int(live.min()) if live.size else -1
    bb = int(ob.bids[:, 0].max())
    return ba, bb


# ---------------------------------------------------------------------------
# CPU oracle of the per-message engine step (``gen_apply``)
# ---------------------------------------------------------------------------

def apply_message_cpu(ob: OrderBook, toks: np.ndarray, tok: MessageTokenizer, p_mid: int, new_oid: int,
                      tick: int = 100, img_levels: int = 500, l2_levels: int = 10, inject=None):
    """Decode one message's tokens, resolve the order id, apply it to ``ob``.

    Returns (raw row (14,), engine msg (8,), provenance, l2 (4*l2_levels,),
    book image (3+img_levels,), new mid)."""
    raw = tok.decode_msgs(np.asarray(toks)[None])[0].astype(np.int64)
    et, dr, price, size = (int(raw[1]), int(raw[2]), int(raw[4]), int(raw[5]))
    ts, tns, tsr, tnsr, pref = (int(raw[8]), int(raw[9]), int(raw[12]), int(raw[13]), int(raw[10]))
    p_abs = p_mid + price * tick
    side = ob.bids if dr == 1 else ob.asks
    hit = np.nonzero((side[:, 4] == tsr) & (side[:, 5] == tnsr))[0]
    oid_l1 = int(side[hit[0], 2]) if hit.size else NEG_RET
    pm = (side[:, 0] == p_abs) & (side[:, 1] > 0)
    if pm.any():
        d = np.abs((side[:, 4] - tsr) * 1000 + np.floor_divide(side[:, 5] - tnsr, 1_000_000))
        d = np.where(pm, d, np.iinfo(np.int32).max)
        oid_l2 = int(side[int(np.argmin(d)), 2])
    else:
        oid_l2 = NEG_RET
    is_cd = et in (2, 3)
    oid_ref = oid_l1 if oid_l1 != NEG_RET else oid_l2
    oid = oid_ref if is_cd else new_oid
    msg = np.array([et, dr * 2 - 1, size, p_abs, oid, -88, ts, tns], dtype=np.int64)
    raw[0], raw[3] = oid, p_abs
    res = 0 if not is_cd else (1 if oid_l1 != NEG_RET else (2 if oid_l2 != NEG_RET else 3))
    prov = res + (8 if is_cd and pref != NA_VAL and price != NA_VAL and price != pref else 0)
    if inject is not None and inject[0]:
        # do(Q): the engine gets our order instead of the generated one (the decoded
        # generated message is still reported in ``raw``)
        msg = np.array([inject[1], inject[2] * 2 - 1, inject[3], p_mid + inject[4] * tick, new_oid, -88, ts, tns],
                       dtype=np.int64)
        prov += 16
    ob.process(msg)
    ba, bb = _best_quotes(ob)
    pm_new = p_mid if (ba <= 0 or bb <= 0) else ((ba + bb) // 2 // tick) * tick
    l2 = ob.l2(l2_levels).astype(np.int64)
    p_change = (pm_new - p_mid) // tick
    img = transform_l2_numpy(np.concatenate([[p_change, ts, tns], l2[:40]]).astype(np.float64), img_levels, tick)
    return raw, msg, prov, l2, img, pm_new


def time_tokens_cpu(msg: torch.Tensor, tok: MessageTokenizer, time: torch.Tensor) -> None:
    """In place: absolute-time tokens of ``msg`` (B, L) from its delta-t tokens; advances ``time`` (B, 2)."""
    off = tok.vocab.codes["time"].offset
    p = tok.FIELD_START["delta_t_s"]
    d = (msg[:, p:p + 4] - off).long()
    dts = d[:, 0]
    dtns = (d[:, 1] * 1000 + d[:, 2]) * 1000 + d[:, 3]
    ns = time[:, 1].long() + dtns
    extra = ns // 1_000_000_000
    ns = ns - extra * 1_000_000_000
    s = time[:, 0].long() + dts + extra
    time[:, 0], time[:, 1] = s.to(time.dtype), ns.to(time.dtype)
    digs = [(s // 1000) % 1000, s % 1000, (ns // 1_000_000) % 1000, (ns // 1000) % 1000, ns % 1000]
    for i, v in enumerate(digs):
        msg[:, p + 4 + i] = off + v


# ---------------------------------------------------------------------------
# state helpers
# ---------------------------------------------------------------------------

def _cat_states(parts):
    if parts[0] is None:
        return None
    if isinstance(parts[0], torch.Tensor):
        return torch.cat(parts, 0)
    return type(parts[0])(_cat_states([p[i] for p in parts]) for i in range(len(parts[0])))


def _assign_state(old, new):
    """Copy ``new`` into ``old`` wherever a step returned a fresh tensor."""
    if old is None:
        return
    if isinstance(old, torch.Tensor):
        if new is not old:
            old.copy_(new)
        return
    for o, n in zip(old, new):
        _assign_state(o, n)


@dataclass
class GenOutput:
    tokens: torch.Tensor      # (B, n, MSG_LEN) int64
    raw: torch.Tensor         # (B, n, 14) int32 decoded messages (order id and abs price filled)
    l2: torch.Tensor          # (B, n, 4*levels) int32 book after each message
    provenance: torch.Tensor  # (B, n) int32 order-id resolution bits
    mid: torch.Tensor         # (B, n) int32 mid price after each message
    engine_msgs: Optional[torch.Tensor] = None   # (B, n, 8) int32 messages the engine processed


class Generator:
    def __init__(self, model, token_mode: str = "22tok", engine_cfg: EngineConfig = EngineConfig(),
                 tick_size: int = 100, top_n: int = -1, img_levels: int = 500, l2_levels: int = 10,
                 seed: int = 0, use_graphs: bool = True, prefill_batch: int = 64):
        self.model, self.tok, self.cfg = model, get_tokenizer(token_mode), engine_cfg
        self.tick, self.top_n, self.img_levels, self.l2_levels = tick_size, top_n, img_levels, l2_levels
        self.seed, self.use_graphs, self.prefill_batch = seed, use_graphs, prefill_batch
        V = getattr(model, "vocab_size", len(self.tok.vocab))
        self.allow_np = syntax_validation_matrix(self.tok, vocab_size=V)
        self.layout = gen_layout(self.tok, tick_size, img_levels, l2_levels)
        self.graph = None

    # -- conditioning ----------------------------------------------------------------------
    @torch.no_grad()
    def condition(self, tokens_in: torch.Tensor, books: torch.Tensor, last_tok: torch.Tensor,
                  l2_start: np.ndarray, engine_msgs: np.ndarray, start_time=(34200, 0)):
        """Prime model and engine with a context.

        tokens_in (B, n_ctx*L) START-shifted context tokens; books (B, n_ctx, d_book)
        per-message book images; last_tok (B,) the context's final token;
        l2_start (B, 4*levels) the book before the context; engine_msgs
        (B, n_ctx, 8) the context as engine messages (replayed into the books)."""
        m = self.model
        dev = next(m.parameters()).device
        self.dev = dev
        if dev.type == "cuda":
            from ..ops import weights as W
            W.freeze(m)
        B = tokens_in.shape[0]
        self.B = B
        L = self.tok.MSG_LEN
        # model: chunked prefill in sub-batches (bounded activation memory)
        parts = []
        for b0 in range(0, B, self.prefill_batch):
            b1 = min(B, b0 + self.prefill_batch)
            st, _ = m.prefill(tokens_in[b0:b1].to(dev), books[b0:b1].to(dev))
            parts.append(st)
        self.state = _cat_states(parts)
        # engine: reset from L2 then replay the context
        self.books_cpu = None
        self.on_gpu = dev.type == "cuda"
        if self.on_gpu:
            from ..ops._ext import ext
            from ..engine.book import init_msgs_from_l2
            c = self.cfg
            self.asks = torch.full((B, c.n_orders, 6), -1, dtype=torch.int32, device=dev)
            self.bids = torch.full_like(self.asks, -1)
            self.trades = torch.full((B, c.n_trades, 8), -1, dtype=torch.int32, device=dev)
            st0 = np.stack([init_msgs_from_l2(np.asarray(r), c, (int(start_time[0]), 0)) for r in l2_start])
            msgs = np.concatenate([st0, np.asarray(engine_msgs)], axis=1).astype(np.int32)
            ext().eng_process(self.asks, self.bids, self.trades, torch.from_numpy(msgs).to(dev), c.init_id,
                              c.book_depth, c.cancel_mode, c.type_4_interpretation, c.check_book_fill)
            l1 = ext().eng_l2(self.asks, self.bids, 1).cpu().numpy()
            ba = np.where(l1[:, 0] == 2147483647, -1, l1[:, 0])
            bb = np.where(l1[:, 2] == -2147483647, -1, l1[:, 2])
        else:
            self.books_cpu = []
            ba, bb = [], []
            for i in range(B):
                ob = book_from_l2(np.asarray(l2_start[i]), self.cfg, (int(start_time[0]), 0))
                ob.process_many(np.asarray(engine_msgs[i]))
                self.books_cpu.append(ob)
                a, b = _best_quotes(ob)
                ba.append(a)
                bb.append(b)
        pm = [safe_mid_price(a, b, self.tick) for a, b in zip(ba, bb)]
        self.p_mid = torch.tensor(pm, dtype=torch.int32, device=dev)
        # running message, time, book input
        last = np.asarray(last_tok.cpu()) if isinstance(last_tok, torch.Tensor) else np.asarray(last_tok)
        ctx_last = np.asarray(tokens_in[:, -(L - 1):].cpu())
        last_msg = np.concatenate([ctx_last, last[:, None]], 1)
        raw = self.tok.decode_msgs(last_msg)
        self.time = torch.tensor(raw[:, 8:10], dtype=torch.int32, device=dev)
        self.msg = torch.zeros(B, L, dtype=torch.int64, device=dev)
        self.msg[:, L - 1] = torch.as_tensor(last, device=dev)
        self.book = books[:, -1:].to(device=dev, dtype=torch.float32).clone()     # (B, 1, d_book), owned
        self.allow = torch.from_numpy(self.allow_np.astype(np.uint8)).to(dev)
        self.ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        self.new_oid = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None
        self._oid_offset = 0
        self._gen = torch.Generator(device=dev).manual_seed(self.seed)

    # -- one message ---------------------------------------------------------------------------
    # -- outside orders ---------------------------------------------------------------------------
    @torch.no_grad()
    def apply_engine_messages(self, msgs) -> torch.Tensor:
        """Process outside orders (B, m, 8) on the generator's books between generated
        messages (a trading agent in the loop); the trades rows are cleared first, so
        the returned (B, n_trades, 8) trades belong to these messages and any generated
        message processed before the next call."""
        msgs = torch.as_tensor(msgs)
        if self.on_gpu:
            from ..ops._ext import ext
            c = self.cfg
            self.trades.fill_(-1)
            ext().eng_process(self.asks, self.bids, self.trades, msgs.to(self.dev, torch.int32).contiguous(),
                              c.init_id, c.book_depth, c.cancel_mode, c.type_4_interpretation, c.check_book_fill)
            return self.trades
        out = []
        for b, ob in enumerate(self.books_cpu):
            ob.trades[:] = -1
            for row in msgs[b].numpy():
                ob.process(row)
            out.append(torch.from_numpy(ob.trades.copy()))
        return torch.stack(out)

    def trade_rows(self) -> torch.Tensor:
        if self.on_gpu:
            return self.trades.cpu().long()
        return torch.from_numpy(np.stack([ob.trades for ob in self.books_cpu]))

    def sides(self):
        if self.on_gpu:
            return self.asks.cpu().long(), self.bids.cpu().long()
        return (torch.from_numpy(np.stack([ob.asks for ob in self.books_cpu])),
                torch.from_numpy(np.stack([ob.bids for ob in self.books_cpu])))

    def _logits(self, h):
        from ..ops import weights as W
        h2 = h[:, -1].to(torch.bfloat16)
        return torch.mm(h2, W.bf16(self.model.decoder.kernel), out_dtype=torch.float32)

    def _sample_into(self, h, pos):
        if self.on_gpu and self.top_n in (1, -1):
            from ..ops._ext import ext
            ext().gen_sample(self._logits(h), self.model.decoder.bias, self.allow[pos], self.seed, self.ctr, pos,
                             self.top_n, self.msg, pos, self.tok.MSG_LEN)
            return
        logits = self.model.decoder(h[:, -1]).float()
        logits = logits.masked_fill(~self.allow[pos].bool(), float("-inf"))
        if self.top_n == 1:
            t = logits.argmax(-1)
        elif self.top_n > 1:
            vals, idx = logits.topk(self.top_n, dim=-1)
            t = idx.gather(-1, torch.multinomial(torch.softmax(vals, -1), 1, generator=self._gen))[:, 0]
        else:
            t = torch.multinomial(torch.softmax(logits, -1), 1, generator=self._gen)[:, 0]
        self.msg[:, pos] = t

    def _model_step(self, col, n=1):
        """Advance the model over message columns col .. col+n-1 (all of them known)."""
        book = self.book if (self.book is None or n == 1) else self.book.expand(-1, n, -1).contiguous()
        st, h = self.model.step_hidden(self.state, self.msg[:, col:col + n], book)
        _assign_state(self.state, st)
        return h

    def _message_device(self):
        """All device work of one message (capturable)."""
        L, ts = self.tok.MSG_LEN, self.tok.TIME_START_I
        for pos in range(ts):
            h = self._model_step((pos - 1) % L)
            self._sample_into(h, pos)
        if self.on_gpu:
            from ..ops._ext import ext
            ext().gen_time_tokens(self.msg, self.tok.FIELD_START["delta_t_s"], self.tok.vocab.codes["time"].offset,
                                  self.time)
        else:
            time_tokens_cpu(self.msg, self.tok, self.time)
        # the previous field's last token and the four computed time tokens go through
        # the model as one 5-token step (no logits are needed for them)
        self._model_step(ts - 1, 5)
        for pos in range(ts + 5, L):
            h = self._model_step(pos - 1)
            self._sample_into(h, pos)
        if self.on_gpu:
            from ..ops._ext import ext
            c = self.cfg
            ext().gen_apply(self.asks, self.bids, self.trades, self.msg, self.layout, c.init_id, c.book_depth,
                            c.cancel_mode, c.type_4_interpretation, c.check_book_fill, self.new_oid, self.p_mid,
                            self.time, self.o_raw, self.o_msg, self.o_prov, self.o_l2, self.book[:, 0], True,
                            self.inj_buf)
            self.ctr.add_(1)
            self.new_oid.sub_(1)

    def _engine_cpu(self, oid: int):
        msg = self.msg.cpu().numpy()
        pm = self.p_mid.cpu().numpy()
        inj = self.inj_buf.cpu().numpy()
        imgs = []
        for b, ob in enumerate(self.books_cpu):
            raw, em, prov, l2, img, pm_new = apply_message_cpu(ob, msg[b], self.tok, int(pm[b]), oid, self.tick,
                                                               self.img_levels, self.l2_levels, inject=inj)
            self.o_raw[b] = torch.from_numpy(raw.astype(np.int32))
            self.o_msg[b] = torch.from_numpy(em.astype(np.int32))
            self.o_l2[b] = torch.from_numpy(l2.astype(np.int32))
            self.o_prov[b] = int(prov)
            pm[b] = pm_new
            imgs.append(img)
        self.p_mid.copy_(torch.from_numpy(pm))
        self.book[:, 0] = torch.from_numpy(np.stack(imgs)).to(self.book.dtype)

    @torch.no_grad()
    def generate(self, n_msgs: int, events=None, inject: Optional[dict] = None) -> GenOutput:
        """Generate ``n_msgs`` messages for every book.

        ``events``: optional list of ``n_msgs + 1`` CUDA events recorded before each
        message and at the end.  ``inject``: do(Q) -- ``{"step": k, "event_type": 1|4,
        "side": 0|1, "qty": Q, "offset_ticks": o}`` replaces the generated order at
        step ``k`` (every book) by that order at ``mid + o`` ticks (the reference's
        ``sample_new`` inject_* arguments, ``docs/inference.md``)."""
        B, L, dev = self.B, self.tok.MSG_LEN, self.dev
        plan = torch.zeros(n_msgs, 5, dtype=torch.int32)
        if inject is not None:
            k = int(inject["step"])
            if not 0 <= k < n_msgs:
                raise ValueError(f"inject step {k} outside the {n_msgs}-message horizon")
            plan[k] = torch.tensor([1, int(inject["event_type"]), int(inject["side"]), int(inject["qty"]),
                                    int(inject.get("offset_ticks", 0))], dtype=torch.int32)
        self.inj_buf = torch.zeros(5, dtype=torch.int32, device=dev)
        self.o_raw = torch.zeros(B, 14, dtype=torch.int32, device=dev)
        self.o_msg = torch.zeros(B, 8, dtype=torch.int32, device=dev)
        self.o_prov = torch.zeros(B, dtype=torch.int32, device=dev)
        self.o_l2 = torch.zeros(B, 4 * self.l2_levels, dtype=torch.int32, device=dev)
        out_tok = torch.zeros(B, n_msgs, L, dtype=torch.int64, device=dev)
        out_raw = torch.zeros(B, n_msgs, 14, dtype=torch.int32, device=dev)
        out_l2 = torch.zeros(B, n_msgs, 4 * self.l2_levels, dtype=torch.int32, device=dev)
        out_prov = torch.zeros(B, n_msgs, dtype=torch.int32, device=dev)
        out_mid = torch.zeros(B, n_msgs, dtype=torch.int32, device=dev)
        out_em = torch.zeros(B, n_msgs, 8, dtype=torch.int32, device=dev)
        # order ids of generated new orders count down within a call (the reference's
        # n_msg_todo) and never repeat across calls
        self.new_oid.fill_(n_msgs + self._oid_offset)
        self.graph = None
        graph = self.on_gpu and self.use_graphs and n_msgs > 1
        for k in range(n_msgs):
            if inject is not None:
                self.inj_buf.copy_(plan[k])
            if events is not None:
                events[k].record()
            if self.on_gpu:
                if graph and self.graph is None and k == 1:
                    self._capture()
                if self.graph is not None:
                    self.graph.replay()
                else:
                    self._message_device()
            else:
                self._message_device()
                self._engine_cpu(n_msgs - k + self._oid_offset)
            out_tok[:, k] = self.msg
            out_raw[:, k] = self.o_raw
            out_l2[:, k] = self.o_l2
            out_prov[:, k] = self.o_prov
            out_mid[:, k] = self.p_mid
            out_em[:, k] = self.o_msg
        if events is not None:
            events[n_msgs].record()
        self._oid_offset += n_msgs
        return GenOutput(out_tok, out_raw, out_l2, out_prov, out_mid, out_em)

    def _capture(self):
        """Capture one message as a CUDA graph (the state buffers are updated in place)."""
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._message_device()
        self.graph = g
