"""Engine utilities: ranking, integer clipping, apportionment, random books/messages, colored noise."""
import numpy as np
import pytest

from sigma0_b200.engine.book import EngineConfig, OrderBook
from sigma0_b200.engine import utils as U


def test_rank_and_clip():
    a = np.array([3, 1, 3, 2])
    assert U.argsort_rev(a).tolist() == [0, 2, 3, 1]
    assert U.rank_rev(a).tolist() == [0, 3, 1, 2]
    assert U.clip_by_sum_int(np.array([3, 2, 3, 1]), 8).tolist() == [3, 2, 2, 1]
    assert U.clip_by_sum_int(np.array([1, 2]), 8).tolist() == [1, 2]
    r = np.random.default_rng(0)
    for _ in range(50):
        v = r.integers(0, 100, 7)
        m = int(r.integers(1, 200))
        c = U.clip_by_sum_int(v, m)
        assert c.sum() == min(m, v.sum()) and (c <= v).all()


def test_hamilton_and_masks():
    s = U.hamilton_apportionment(np.array([10, 10, 10]), 4, np.random.default_rng(1))
    assert s.sum() == 4 and sorted(s.tolist()) == [1, 1, 2]
    s2 = U.hamilton_apportionment(np.array([50, 30, 20]), 10)
    assert s2.tolist() == [5, 3, 2]
    ma, mc = U.matching_masks(np.array([5, 0, 7]), np.array([7, 0, 9]))
    assert ma.tolist() == [False, False, True] and mc.tolist() == [True, False, False]


def test_random_books_and_messages_drive_the_engine():
    rng = np.random.default_rng(2)
    cfg = EngineConfig()
    asks, bids, trades = U.create_init_book(cfg, order_capacity=10, rng=rng)
    assert (asks[:5, 2] == [-2, -4, -6, -8, -10]).all() and (asks[5:] == -1).all() and (trades == -1).all()
    d, m = U.create_message("limit", "ask", 2200100, 5, 36000, 1, 77)
    assert m.tolist() == [1, -1, 5, 2200100, 77, 77, 36000, 1] and d["side"] == -1
    with pytest.raises(ValueError):
        U.create_message("bogus")
    _, c = U.get_random_order_to_cancel(bids, "bid", rng=rng)
    assert c[0] == 2 and c[4] in bids[:, 2]
    _, agg = U.get_random_aggressive_order(asks, "ask", rng=rng)
    live = asks[asks[:, 2] != -1]
    assert agg[1] == 1 and agg[3] == live[:, 0].min()
    ob = OrderBook(cfg)
    ob.process(U.create_message("limit", "ask", 2200100, 10, 36000, 0, 1)[1])
    ob.process(U.create_message("limit", "bid", 2200100, 4, 36000, 1, 2)[1])
    assert (ob.trades[:, 0] != -1).sum() == 1


@pytest.mark.parametrize("beta", [0.0, 1.0, 2.0])
def test_powerlaw_noise_spectrum_and_variance(beta):
    x = U.powerlaw_psd_gaussian(beta, (400, 1024), np.random.default_rng(3))
    assert abs(x.var() - 1.0) < 0.15
    p = (np.abs(np.fft.rfft(x, axis=-1)) ** 2).mean(0)[1:]
    f = np.fft.rfftfreq(1024)[1:]
    slope = np.polyfit(np.log(f[5:400]), np.log(p[5:400]), 1)[0]
    assert abs(slope + beta) < 0.15
