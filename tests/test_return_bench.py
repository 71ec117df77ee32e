"""The event-anchored return bench: each rule that would change answers silently when
broken is pinned by a case that fails under the broken version, and the bench on a
generation run scores the real stream fed in as generated with IC exactly 1."""
import numpy as np
import pandas as pd
import pytest

from sigma0_b200.eval import return_bench as R


def test_price_at_horizon_rules():
    t = np.array([10.0, 10.001, 10.002, 10.002, 10.005])
    m = np.array([100.0, 101.0, 102.0, 103.0, 104.0])
    # past the end of the stream: not covered (not the last row)
    assert R.price_at(t, m, 10.0, 99.0, 6.0)[0] is False
    # messages sharing the target time count: the LAST one at or before it
    assert R.price_at(t, m, 10.0, 99.0, 2.0) == (True, 103.0)
    # no look-ahead: between messages the earlier row holds
    assert R.price_at(t, m, 10.0, 99.0, 4.0) == (True, 103.0)
    # nothing by then: the anchor's mid
    assert R.price_at(t, m, 9.0, 99.0, 0.5) == (True, 99.0)


def test_pairs_need_both_streams_and_skill_numbers():
    g = R.anchored_returns([1.0, 10.0], 0.0, 100.0, np.array([0.0005, 0.02]), np.array([101.0, 102.0]),
                           np.array([0.0008, 0.005]), np.array([99.0, 98.0]))
    assert list(g) == [1.0]                                  # 10 ms: the real stream ended at 5 ms
    assert g[1.0] == pytest.approx((np.log(1.01), np.log(0.99)))
    pred = np.array([0.1, -0.2, 0.3, 0.0, 0.5])
    s = R.skill(pred, pred.copy())
    assert s["IC"] == pytest.approx(1.0) and s["ranked_IC"] == pytest.approx(1.0) and s["N_eff"] == 4
    assert R.skill(pred, -pred)["direction_acc"] == 0.0
    assert R.trade_sign_baseline([1, -1]).tolist() == [-1.0, 1.0]


def _run_dir(tmp_path, n_windows=24, nc=60, ng=80):
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.sim.divergence import run_paths
    d = make_sequences(1, 4000, seed=11)[0]
    em = np.asarray(d.engine_msgs, np.int64)
    after = np.asarray(d.books[1:, 3:], np.int64)          # the book after message i
    root = str(tmp_path / "run")
    for sub in ("data_cond", "data_real", "data_gen"):
        (tmp_path / "run" / sub).mkdir(parents=True)

    def write_msgs(path, m):
        pd.DataFrame({"time": [f"{s}.{ns:09d}" for s, ns in m[:, 6:8]], "event_type": m[:, 0],
                      "order_id": m[:, 4], "size": m[:, 2], "price": m[:, 3], "direction": m[:, 1]}).to_csv(
            path, index=False)
    trades = [i for i in range(nc, len(em) - ng - 1) if em[i, 0] == 4]
    rng = np.random.default_rng(0)
    picks = sorted(rng.choice(trades, n_windows, replace=False))
    for k, i in enumerate(picks):
        s = i - nc + 1                                      # the window's last conditioning message is a trade
        p = run_paths(root, "SYN", "2000-01-01", k)
        write_msgs(p["cond_msg"], em[s:i + 1])
        pd.DataFrame(after[s - 1:i + 1]).to_csv(p["cond_book"], index=False)
        write_msgs(p["real_msg"], em[i + 1:i + 1 + ng])
        pd.DataFrame(after[i + 1:i + 1 + ng]).to_csv(p["real_book"], index=False)
        # "generated": another stretch of the day, moved onto this window's clock and price level
        j = int(rng.integers(nc, len(em) - ng - 1))
        g = em[j + 1:j + 1 + ng].copy()
        shift_ns = (em[i, 6] * 10**9 + em[i, 7]) - (em[j, 6] * 10**9 + em[j, 7])
        tns = g[:, 6] * 10**9 + g[:, 7] + shift_ns
        g[:, 6], g[:, 7] = tns // 10**9, tns % 10**9
        write_msgs(p["gen_msg"], g)
        gb = after[j + 1:j + 1 + ng].copy()
        lvl = (after[i, 0] + after[i, 2]) // 2 - (after[j, 0] + after[j, 2]) // 2
        gb[:, 0::2] += lvl
        pd.DataFrame(gb).to_csv(p["gen_book"], index=False)
    return root


def test_return_bench_on_a_generation_run(tmp_path):
    root = _run_dir(tmp_path)
    wins = R.load_run(root, "SYN")
    assert len(wins) == 24
    ident = R.bench(wins, [5.0, 50.0], identity=True, n_null=20)
    assert ident["windows_used"] == 24
    for v in ident["horizons"].values():
        if v["N"] >= 3:
            assert v["IC"] == pytest.approx(1.0, abs=1e-12) and v["gen_msgs_mean"] == v["real_msgs_mean"]
    res = R.bench(wins, [5.0, 50.0], n_null=20)
    for v in res["horizons"].values():
        if v["N"] >= 3:
            assert -1.0 <= v["IC"] <= 1.0 and "trade_sign_baseline" in v and "IC_mean" in v["null"]
    assert R.main(["--run_dir", root, "--identity_check", "--horizons_ms", "5", "50"]) == 0
