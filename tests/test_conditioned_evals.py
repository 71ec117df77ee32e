"""Tail-, regime- and position-conditioned breakdowns (eval/conditioned.py) on synthetic
windows with known answers."""
import numpy as np
import pytest

from sigma0_b200.eval import conditioned as C


def test_w1_shift_and_identity():
    rng = np.random.default_rng(0)
    a = rng.standard_normal(20000)
    assert C.w1(a, a) == pytest.approx(0.0, abs=1e-12)
    assert C.w1(a, a + 0.7) == pytest.approx(0.7, rel=1e-6)


def test_tail_conditioned_flags_a_heavier_generated_tail():
    rng = np.random.default_rng(1)
    r = rng.standard_normal(50000)
    g_same = rng.standard_normal(50000)
    g_heavy = rng.standard_t(3, 50000)
    same = C.tail_conditioned({"x": r}, {"x": g_same})["features"]["x"]
    heavy = C.tail_conditioned({"x": r}, {"x": g_heavy})["features"]["x"]
    assert same["ws_bulk"] < 0.03 and same["qratio_0.99"] == pytest.approx(1.0, abs=0.1)
    assert heavy["ratio_0.99_norm"] > 1.0 and heavy["qratio_0.99"] > 1.2
    assert heavy["n_real_tail_0.9"] == pytest.approx(5000, abs=2)


def _window(rng, n, drift):
    mid = 10000 * 100 + np.cumsum(rng.integers(-1, 2, n) * 100) + drift * np.arange(n) * 100
    sp = 100 * (rng.integers(1, 3, n) + rng.integers(0, 6))     # each window its own spread level
    book = np.stack([mid + sp // 2, rng.integers(1, 50, n), mid - sp // 2, rng.integers(1, 50, n)], 1)
    t = np.cumsum(rng.exponential(0.01, n))
    msgs = np.stack([np.floor(t), (t % 1) * 1e9, rng.integers(1, 5, n), np.arange(n), rng.integers(1, 100, n),
                     mid, rng.choice([-1, 1], n)], 1)
    return msgs, book


def test_regime_ic_is_one_for_a_perfect_generator():
    rng = np.random.default_rng(2)
    wins = [_window(rng, 120, d) for d in rng.normal(0, 0.3, 60)]
    msgs = [w[0] for w in wins]
    books = [w[1] for w in wins]
    res = C.run_all(msgs, books, msgs, books, bin_width=30)
    for strat in ("spread", "volatility"):
        for t in ("low", "mid", "high"):
            blk = res["regime"]["data"][strat][t]
            assert blk["n"] > 0 and blk["ic"] == pytest.approx(1.0) and blk["ws"] == pytest.approx(0.0, abs=1e-9)
    assert all(v == pytest.approx(0.0, abs=1e-9) for v in res["position"]["ws_tau"])
    assert set(res["tail"]["features"]) >= {"spread", "ofi", "orderbook_imbalance"}


def test_position_drift_and_fit():
    rng = np.random.default_rng(3)
    n_win, L = 200, 200
    real = rng.standard_normal((n_win, L))
    tau = np.arange(L)
    gen = rng.standard_normal((n_win, L)) + 0.002 * tau[None, :] ** 1.5     # drift grows with position
    res = C.position_in_window({"spread": real}, {"spread": gen}, bin_width=20, features=("spread",), c=100)
    ws = np.array(res["ws_tau"])
    assert ws[-1] > ws[0] + 0.3
    fit = res["fit_single_c"]
    assert fit["beta"] > 0 and 1.0 < fit["p"] < 2.2
    t = np.linspace(5, 200, 12)
    exact = C.fit_power_curve(t, 0.1 + 0.02 * t ** 1.3)
    assert exact["alpha"] == pytest.approx(0.1, abs=1e-3) and exact["p"] == pytest.approx(1.3, abs=1e-3)


def test_cg_surface_c_star():
    runs = [{"c": c, "fit_single_c": {"alpha": a}} for c, a in ((0, 1.0), (50, 0.5), (100, 0.12), (200, 0.05),
                                                                (400, 0.04))]
    res = C.fit_cg_surface(runs)
    assert res["alpha_0"] == 1.0 and res["alpha_cmax"] == 0.04
    assert res["c_star"] == 100.0


def test_dense_features_basic_values():
    msgs = np.array([[0, 0, 1, 1, 10, 9900, 1], [0, 5e8, 1, 2, 5, 10300, -1], [1, 0, 3, 1, 10, 9900, 1]], float)
    book = np.array([[10100, 7, 9900, 3], [10100, 7, 9900, 3], [10100, 7, 9800, 4]], float)
    f = C.dense_features(msgs, book)
    np.testing.assert_allclose(f["spread"], [2, 2, 3])
    np.testing.assert_allclose(f["ofi"], [10, -5, -10])
    np.testing.assert_allclose(f["limit_bid_order_depth"][0], 0.0)
    np.testing.assert_allclose(f["limit_ask_order_depth"][1], 2.0)
    assert np.isnan(f["log_inter_arrival_time"][0]) and f["log_inter_arrival_time"][1] == pytest.approx(np.log(0.5))


def test_observational_comparisons_on_identical_runs():
    from sigma0_b200.eval import observational as O
    rng = np.random.default_rng(4)
    wins = [_window(rng, 300, d) for d in rng.normal(0, 0.3, 40)]
    msgs, books = [w[0] for w in wins], [w[1] for w in wins]
    j = O.joint_canonical(msgs, books, msgs, books)
    assert j["delta_rho"] == pytest.approx(0.0) and j["closure"] == pytest.approx(1.0)
    assert j["sliced_w2"] == pytest.approx(0.0, abs=1e-9) and j["sliced_w2_floor_real_vs_real"] > 0
    otm = O.otm_observational(msgs, books, msgs, books, H=20)
    assert otm["R_real"] == otm["R_gen"] and sum(v[1] for v in otm["R_real"].values()) > 0
    r = rng.standard_normal(20000)
    base = O.resampler_baseline({"x": r}, {"x": r + 2.0})["resampler_gap_closure"]["x"]
    assert base["ws_model"] == pytest.approx(2.0, rel=1e-3) and base["gap_closure"] < -10
    rep = O.reproducibility({"x": 0.1, "y": 0.2}, {"x": 0.12})
    assert rep["per_feature"] == {"x": {"this": 0.1, "baseline": 0.12}}
    assert O.reproducibility({"x": 0.1}, None)["status"] == "no baseline available"
