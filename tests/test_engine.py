"""CPU order-book engine: the reference smoke vectors (tests/smoke/test_matching_engine.py)
plus cancel, eviction and IOC semantics."""
import numpy as np

from sigma0_b200.engine import OrderBook, EngineConfig, book_from_l2, MAXINT, init_msgs_from_l2

L2_INIT = [354200, 452, 350100, 89, 361200, 100, 344000, 400, 362900, 100,
           343100, 100, 364000, 400, 338700, 100, 371900, 1100, 337100, 1000]
BEST_ASK, BEST_ASK_QTY = 354200, 452
BEST_BID, BEST_BID_QTY = 350100, 89


def book():
    return book_from_l2(np.array(L2_INIT))


def test_reset_top_of_book():
    ob = book()
    bid, ask = ob.best_bid_ask()
    assert ask[0] == BEST_ASK and ask[1] == BEST_ASK_QTY
    assert bid[0] == BEST_BID and bid[1] == BEST_BID_QTY


def test_l2_shape_and_values():
    l2 = book().l2(4)
    assert l2.shape == (16,)
    assert l2[0] == BEST_ASK and l2[1] == BEST_ASK_QTY and l2[2] == BEST_BID
    full = book().l2(10)
    assert full[4 * 5] == MAXINT and full[4 * 5 + 1] == 0 and full[4 * 5 + 2] == -MAXINT


def test_crossing_bid_trades_and_consumes():
    ob = book()
    ob.process([1, 1, 100, 355000, 7777, 7777, 3402, 1000])
    assert ob.best_bid_ask()[1][0] == BEST_ASK
    assert ob.l2(1)[1] == BEST_ASK_QTY - 100
    filled = ob.trades[(ob.trades != -1).any(axis=1)]
    assert filled.shape[0] == 1
    assert filled[0, 0] == BEST_ASK and abs(filled[0, 1]) == 100
    assert 7777 in (filled[0, 3], filled[0, 7])


def test_non_crossing_bid_rests():
    ob = book()
    ob.process([1, 1, 50, 351000, 6666, 6666, 3403, 2000])
    assert ob.best_bid_ask()[0][0] == 351000
    assert int((ob.trades != -1).any(axis=1).sum()) == 0


def test_cancel_by_id_then_init_fallback():
    ob = book()
    ob.process([1, -1, 30, 360000, 55, 0, 34201, 0])
    ob.process([2, -1, 10, 360000, 55, 0, 34202, 0])
    assert ob.asks[ob.asks[:, 2] == 55, 1][0] == 20
    ob.process([3, -1, 20, 360000, 55, 0, 34203, 0])
    assert not (ob.asks[:, 2] == 55).any()
    # unknown id at an init level: falls back to the init order there
    ob.process([2, 1, 9, BEST_BID, 999, 0, 34204, 0])
    assert ob.l2(1)[3] == BEST_BID_QTY - 9


def test_execution_is_ioc():
    ob = book()
    # execute 500 against the best bid (89): fills 89 at best bid, then 400 at 344000, rest discarded
    ob.process([4, 1, 500, 340000, -3, 0, 34210, 0])
    l2 = ob.l2(3)
    assert l2[2] == 343100   # bids at 350100 and 344000 consumed
    assert not (ob.asks[:, 2] == -3).any()   # nothing rested on the ask side


def test_full_side_evicts_worst():
    cfg = EngineConfig(n_orders=4)
    ob = OrderBook(cfg)
    for k, p in enumerate([100, 101, 102, 103]):
        ob.process([1, 1, 1, p, k + 1, 0, 34200, k])
    ob.process([1, 1, 1, 99, 9, 0, 34200, 9])   # side full -> evict worst (100) then add
    assert 100 not in ob.bids[:, 0] and 99 in ob.bids[:, 0]


def test_init_msgs_layout():
    m = init_msgs_from_l2(np.array(L2_INIT))
    assert m.shape == (10, 8)
    assert (m[0::2, 1] == -1).all() and (m[1::2, 1] == 1).all()
    assert m[0, 4] == -2 and m[1, 4] == -3
