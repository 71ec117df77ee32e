"""Generator metrics against the real continuation: book losses compare by price, so one
added level is one difference, and the Wasserstein distance of normalised profiles; return
correlation, moments, liquidity and event counts."""
import numpy as np
import pytest

from sigma0_b200.eval import gen_metrics as G

E = 2 ** 31 - 1


def _book(asks, bids, levels=3):
    row = []
    for i in range(levels):
        ap, av = asks[i] if i < len(asks) else (E, 0)
        bp, bv = bids[i] if i < len(bids) else (-E, 0)
        row += [ap, av, bp, bv]
    return np.array(row)


def test_book_losses_compare_by_price():
    real = _book([(101, 10), (102, 20), (103, 5)], [(100, 7), (99, 3), (98, 4)])
    assert G.book_loss_l1(real, real) == 0.0 and G.book_loss_wasserstein(real, real) == 0.0
    # the best bid removed: every bid level shifts up in a positional comparison, by price one
    # price differs (plus the level that moved into view at the bottom edge)
    gen = _book([(101, 10), (102, 20), (103, 5)], [(99, 3), (98, 4), (97, 9)])
    vg, vr = G.compared_volumes(gen, real, 3)
    assert len(vg) == 7 and int(np.count_nonzero(vg - vr)) == 2
    assert G.book_loss_l1(gen, real) == pytest.approx((7 + 9) / 7)
    assert G.book_loss_wasserstein(gen, real) > 0
    # one share moved by one price step costs less than moved by two (normalised profiles)
    one = _book([(101, 10), (102, 20), (103, 5)], [(100, 6), (99, 4), (98, 4)])
    two = _book([(101, 10), (102, 20), (103, 5)], [(100, 6), (99, 3), (98, 5)])
    assert G.book_loss_wasserstein(one, real) < G.book_loss_wasserstein(two, real)


def test_returns_moments_liquidity_events():
    rng = np.random.default_rng(0)
    r = rng.standard_normal((50, 4))
    assert np.allclose(G.return_corr(r, r), 1.0) and np.allclose(G.return_corr(r, -r), -1.0)
    lo, hi = G.return_corr_ci(r, r + 0.1 * rng.standard_normal(r.shape), n_boot=50)
    assert (lo <= hi).all() and (hi <= 1.0 + 1e-12).all()
    m = G.moments(rng.standard_normal(20000))
    assert abs(m["mean"]) < 0.05 and abs(m["std"] - 1) < 0.05 and abs(m["excess_kurtosis"]) < 0.2
    ci = G.moments_ci(rng.standard_normal(500), n_boot=50)
    assert all(lo < hi for lo, hi in ci.values())
    msgs = np.zeros((5, 14), np.int64)
    msgs[:, 1] = [1, 1, 3, 4, 2]
    msgs[:, 5] = [10, 20, 5, 7, 1]
    prov, taken = G.liquidity(msgs)
    assert prov.tolist() == [10, 30, 30, 30, 30] and taken.tolist() == [0, 0, 5, 12, 13]
    assert G.event_type_counts(msgs) == {1: 2, 2: 1, 3: 1, 4: 1}


def test_evaluate_on_a_generated_and_real_path():
    from sigma0_b200.data.synthetic import make_sequences
    d = make_sequences(1, 400, seed=2)[0]
    b = np.asarray(d.books[:, 3:], np.int64)
    W, S = 6, 20
    real = np.stack([b[w * 50 + 1:w * 50 + 1 + S] for w in range(W)])
    gen = np.stack([b[w * 50 + 2:w * 50 + 2 + S] for w in range(W)])     # one message out of step
    rm = np.stack([d.msgs[w * 50:w * 50 + S] for w in range(W)])
    mid0 = (b[[w * 50 for w in range(W)], 0] + b[[w * 50 for w in range(W)], 2]) / 2
    res = G.evaluate(gen, real, rm, rm, mid0, n_boot=20)
    assert len(res["book_loss_l1"]) == S and np.isfinite(res["book_loss_l1"]).all()
    assert res["events_gen"] == res["events_real"]
    same = G.evaluate(real, real, rm, rm, mid0, n_boot=20)
    assert max(same["book_loss_l1"]) == 0.0 and max(same["mid_loss_l1_ticks"]) == 0.0


def test_gen_metrics_on_a_generation_run(tmp_path):
    """The metrics over a run written by the generation CLI."""
    from sigma0_b200.cli.infer import main
    out = str(tmp_path / "run")
    assert main(["--preset", "smoke", "--impl", "torch", "--synthetic", "3", "--n_sequences", "3", "--batch_size", "3",
                 "--n_cond_msgs", "4", "--n_gen_msgs", "6", "--sample_top_n", "1", "--save_dir", out]) == 0
    res = G.evaluate_run(out, "SYN", n_boot=10)
    assert res["n_windows"] == 3 and res["n_steps"] == 6 and len(res["book_loss_l1"]) == 6
    assert sum(res["events_gen"].values()) == 18 and sum(res["events_real"].values()) == 18
    assert G.main(["--run_dir", out, "--n_boot", "5"]) == 0
