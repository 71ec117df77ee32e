"""Engine utilities: random books and messages, integer apportionment, colored noise.

The helpers of the reference's ``matching_engine/utils/utils.py:11-272`` and
``utils/colorednoise.py:12``, for the numpy engine (``engine/book.py``) and tests:

* ``argsort_rev`` / ``rank_rev`` -- descending order / rank with left-to-right
  priority among ties;
* ``clip_by_sum_int`` -- scale a non-negative integer vector down to sum at most
  ``max_sum`` keeping proportions (largest remainders get the leftover units, ties
  left to right); e.g. [3, 2, 3, 1] with 8 -> [3, 2, 2, 1];
* ``hamilton_apportionment`` -- Hamilton (largest remainder) seat allocation with
  ties among the largest remainders broken at random;
* ``matching_masks`` -- which of two price lists' entries occur in the other
  (price 0 never matches);
* ``create_init_book``, ``create_message``, ``create_rand_message``,
  ``get_random_order_to_cancel``, ``get_random_aggressive_order`` -- book sides and
  engine message rows ``[type, side, qty, price, oid, tid, sec, ns]`` for tests;
* ``powerlaw_psd_gaussian`` -- unit-variance Gaussian noise with power spectrum
  proportional to ``f ** -exponent`` (Timmer & Koenig, A&A 300, 707, 1995: random
  Fourier amplitudes and phases scaled by the target spectrum, inverse real FFT).
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple, Union

import numpy as np

from .book import EMPTY, EngineConfig

LIMIT, CANCEL, MATCH = 1, 2, 4
BID, ASK = 1, -1
DUMMYID = -888_888
STARTOFDAY = (34200, 0)
NS_PER_SEC = 1_000_000_000


def argsort_rev(a: np.ndarray) -> np.ndarray:
    """Indices of ``a`` in descending order; equal values keep left-to-right order."""
    a = np.asarray(a)
    return np.lexsort((np.arange(len(a)), -a)) if a.dtype.kind in "iuf" else np.argsort(-a, kind="stable")


def rank_rev(a: np.ndarray) -> np.ndarray:
    """Rank of each entry in descending order (0 = largest; ties: leftmost first)."""
    r = np.empty(len(a), dtype=np.int64)
    r[argsort_rev(a)] = np.arange(len(a))
    return r


def clip_by_sum_int(a: np.ndarray, max_sum: int) -> np.ndarray:
    a = np.asarray(a, dtype=np.int64)
    total = int(a.sum())
    if total <= max_sum:
        return a.copy()
    base, rem = np.divmod(a * max_sum, total)
    rest = max_sum - int(base.sum())
    return base + (rank_rev(rem) < rest)


def hamilton_apportionment(votes: np.ndarray, seats: int, rng: Optional[np.random.Generator] = None) -> np.ndarray:
    rng = rng or np.random.default_rng()
    v = np.asarray(votes, dtype=np.float64)
    quota = v * seats / v.sum()
    out = np.floor(quota).astype(np.int64)
    rem = quota - out
    for _ in range(seats - int(out.sum())):
        best = np.flatnonzero(rem == rem.max())
        i = int(rng.choice(best))
        out[i] += 1
        rem[i] = -1.0
    return out


def matching_masks(prices_a: np.ndarray, prices_cnl: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """(which prices_a occur in prices_cnl, which prices_cnl occur in prices_a), 0 excluded."""
    pa, pc = np.asarray(prices_a), np.asarray(prices_cnl)
    eq = (pa[:, None] == pc[None, :]) & (pa[:, None] != 0)
    return eq.any(1), eq.any(0)


def create_init_book(cfg: EngineConfig = EngineConfig(), order_capacity: int = 10, trade_capacity: int = 10,
                     pricerange: Sequence[int] = (2190000, 2200000, 2210000), quantrange: Sequence[int] = (0, 500),
                     timeinit: Sequence[int] = STARTOFDAY, percent_fill: float = 0.5,
                     rng: Optional[np.random.Generator] = None):
    """(asks, bids, trades): ``percent_fill`` of each side filled with uniform random init
    orders (asks in [mid, hi], bids in [lo, mid]), init ids counting down from cfg.init_id."""
    rng = rng or np.random.default_rng()
    n = int(order_capacity * percent_fill)
    asks = np.full((order_capacity, 6), EMPTY, dtype=np.int64)
    bids = np.full((order_capacity, 6), EMPTY, dtype=np.int64)
    oid = cfg.init_id
    for i in range(n):
        asks[i] = [rng.integers(pricerange[1], pricerange[2] + 1), rng.integers(quantrange[0], quantrange[1] + 1),
                   oid, oid, timeinit[0], timeinit[1]]
        bids[i] = [rng.integers(pricerange[0], pricerange[1] + 1), rng.integers(quantrange[0], quantrange[1] + 1),
                   oid - 1, oid - 1, timeinit[0], timeinit[1]]
        oid -= 2
    trades = np.full((trade_capacity, 8), EMPTY, dtype=np.int64)
    return asks, bids, trades


def create_message(type: str = "limit", side: str = "bid", price: int = 2200000, quant: int = 10,
                   times: int = 36000, timens: int = 0, id: int = 8888):
    """(dict, engine row) of one message; ``type`` limit / cancel / delete / market."""
    types = {"limit": LIMIT, "cancel": CANCEL, "delete": CANCEL, "market": MATCH}
    sides = {"bid": BID, "ask": ASK}
    if type not in types:
        raise ValueError("type must be one of limit, cancel, delete, market")
    if side not in sides:
        raise ValueError("side must be bid or ask")
    t, s = types[type], sides[side]
    d = {"side": s, "type": t, "price": price, "quantity": quant, "orderid": id, "traderid": id,
         "time": times, "time_ns": timens}
    return d, np.array([t, s, quant, price, id, id, times, timens], dtype=np.int64)


def create_rand_message(type: Optional[str] = "limit", side: Optional[str] = None,
                        price_range=(2100000, 2200000), quant_range=(0, 500), prev_time=STARTOFDAY,
                        times_range=(0, 2), timens_range=(0, NS_PER_SEC), rng=None):
    rng = rng or np.random.default_rng()
    type = type or str(rng.choice(["limit", "cancel", "market"]))
    side = side or str(rng.choice(["bid", "ask"]))
    return create_message(type, side, int(rng.integers(price_range[0], price_range[1] + 1)),
                          int(rng.integers(quant_range[0], quant_range[1] + 1)),
                          prev_time[0] + int(rng.integers(times_range[0], times_range[1] + 1)),
                          prev_time[1] + int(rng.integers(timens_range[0], timens_range[1] + 1)))


def get_random_order_to_cancel(book_side: np.ndarray, side: str = "bid", prev_time=(44444, 44444),
                               times_range=(0, 2), timens_range=(0, NS_PER_SEC), rng=None):
    """A cancel message for a uniformly chosen resting order of ``book_side``."""
    rng = rng or np.random.default_rng()
    live = book_side[book_side[:, 2] != EMPTY]
    if len(live) == 0:
        raise ValueError("no resting order to cancel")
    o = live[int(rng.integers(0, len(live)))]
    return create_message("cancel", side, int(o[0]), int(o[1]),
                          prev_time[0] + int(rng.integers(times_range[0], times_range[1] + 1)),
                          prev_time[1] + int(rng.integers(timens_range[0], timens_range[1] + 1)), int(o[2]))


def get_random_aggressive_order(book_side: np.ndarray, side: str = "bid", prev_time=(44444, 44444),
                                times_range=(0, 2), timens_range=(0, NS_PER_SEC), rng=None):
    """A limit order on the opposite side at ``book_side``'s best price, for a random
    quantity in [0, 2 x the volume there]: it is guaranteed to cross."""
    rng = rng or np.random.default_rng()
    live = book_side[book_side[:, 2] != EMPTY]
    if len(live) == 0:
        raise ValueError("the side is empty")
    best = int(live[:, 0].max() if side == "bid" else live[:, 0].min())
    vol = int(live[live[:, 0] == best, 1].sum())
    return create_message("limit", "ask" if side == "bid" else "bid", best, int(rng.integers(0, 2 * vol + 1)),
                          prev_time[0] + int(rng.integers(times_range[0], times_range[1] + 1)),
                          prev_time[1] + int(rng.integers(timens_range[0], timens_range[1] + 1)), DUMMYID)


def powerlaw_psd_gaussian(exponent: float, size: Union[int, Sequence[int]], rng=None,
                          fmin: float = 0.0) -> np.ndarray:
    """Gaussian noise with S(f) ~ f**-exponent along the last axis, unit variance."""
    rng = rng or np.random.default_rng()
    shape = (size,) if isinstance(size, (int, np.integer)) else tuple(size)
    n = shape[-1]
    f = np.fft.rfftfreq(n)
    fmin = max(fmin, 1.0 / n)
    fc = np.where(f < fmin, fmin, f)
    amp = fc ** (-exponent / 2.0)
    # expected variance of the series built below: the DC (and, for even n, Nyquist) bins
    # are real with variance 2 amp^2, every other bin contributes 4 amp^2
    var = 2.0 * amp[0] ** 2 + 4.0 * np.sum(amp[1:] ** 2)
    if n % 2 == 0:
        var -= 2.0 * amp[-1] ** 2
    sigma = np.sqrt(var) / n
    lead = shape[:-1] + (len(f),)
    re = rng.standard_normal(lead) * amp
    im = rng.standard_normal(lead) * amp
    if n % 2 == 0:
        im[..., -1] = 0.0
        re[..., -1] *= np.sqrt(2.0)
    im[..., 0] = 0.0
    re[..., 0] *= np.sqrt(2.0)
    return np.fft.irfft(re + 1j * im, n=n, axis=-1) / sigma
