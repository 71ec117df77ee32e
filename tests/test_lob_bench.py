"""LOB-Bench scoring (``eval/lob_bench.py``) and the Cont-Stoikov-Talreja baseline
(``eval/cst.py``) on synthetic order flow, CPU."""
import numpy as np
import pytest

from sigma0_b200.data.synthetic import make_sequences
from sigma0_b200.eval import cst, lob_bench


def _streams(n, length, seed):
    out_m, out_b = [], []
    for d in make_sequences(n, length, seed=seed):
        em = d.engine_msgs
        # engine rows (type, side, size, price, oid, trader, time_s, time_ns) -> scorer rows
        m = np.stack([em[:, 6], em[:, 7], em[:, 0], em[:, 4], em[:, 2], em[:, 3], em[:, 1]], 1)
        out_m.append(m)
        out_b.append(np.asarray(d.books[:, 3:], np.int64))
    return out_m, out_b


def test_every_unconditional_metric_is_computed():
    m, b = _streams(3, 600, 1)
    vals = lob_bench.compute(m, b)
    assert len(lob_bench.METRICS) == 22 and set(vals) == set(lob_bench.METRICS)
    for k in ("spread", "orderbook_imbalance", "log_inter_arrival_time", "ask_volume_touch", "bid_volume",
              "limit_ask_order_depth", "limit_bid_order_ticks", "ofi"):
        assert len(vals[k]) > 0 and np.isfinite(vals[k]).all(), k
    assert (vals["spread"] >= 1).all()


def test_same_process_scores_closer_than_a_different_one():
    real_m, real_b = _streams(3, 800, 1)
    same_m, same_b = _streams(3, 800, 2)            # the same generator, other seeds
    p = cst.CSTParams(k=2.0, alpha=0.3, mu=0.5, theta=np.full(10, 0.5), tick=100, unit=100)
    cst_m, cst_b = zip(*[cst.simulate(p, 800, seed=s, mid0=1_000_000) for s in range(3)])
    r = lob_bench.compute(real_m, real_b)
    s1 = {x.metric: x.value for x in lob_bench.score_unconditional(lob_bench.compute(same_m, same_b), r, n_boot=0)
          if x.distance == "l1"}
    s2 = {x.metric: x.value for x in lob_bench.score_unconditional(lob_bench.compute(list(cst_m), list(cst_b)), r,
                                                                   n_boot=0) if x.distance == "l1"}
    common = [k for k in s1 if np.isfinite(s1[k]) and np.isfinite(s2.get(k, np.nan))]
    assert np.mean([s1[k] for k in common]) < np.mean([s2[k] for k in common])


def test_conditional_and_impact_scores():
    real_m, real_b = _streams(2, 800, 3)
    gen_m, gen_b = _streams(2, 800, 4)
    res = lob_bench.run_bench(gen_m, gen_b, real_m, real_b, n_boot=5)
    names = {x.metric for x in res["conditional"]}
    assert names == set(lob_bench.COND_METRICS)
    assert all(np.isfinite(x.value) for x in res["conditional"])
    assert np.isfinite(res["impact"]["mean"])
    resp = lob_bench.impact_responses(real_m, real_b)
    assert set(resp) == {"MO0", "MO1", "LO0", "LO1", "CA0", "CA1"}


def test_cst_simulation_is_a_valid_book_and_estimation_recovers_rates():
    p = cst.CSTParams(k=3.0, alpha=0.6, mu=1.0, theta=np.full(10, 0.3), tick=100, unit=100)
    m, b = cst.simulate(p, 6000, seed=0)
    ok = (b[:, 0] < 2e9) & (b[:, 2] > -2e9)
    assert ok.all() and (b[ok, 0] > b[ok, 2]).all()          # never crossed, never one-sided
    assert (m[:, 5] % 100 == 0).all() and np.isin(m[:, 2], (1, 3, 4)).all()
    est = cst.estimate(m, b)
    assert est.mu == pytest.approx(p.mu, rel=0.3)
    assert est.k == pytest.approx(p.k, rel=0.3)
    assert est.alpha == pytest.approx(p.alpha, abs=0.25)
