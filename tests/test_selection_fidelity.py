"""Checkpoint selection (iso-CE, convergence) and the simulator's replay-fidelity arms, CPU."""
import numpy as np
import pytest

from sigma0_b200.train.checkpoint_selection import convergence_step, select_checkpoints


def test_select_best_and_iso_ce():
    rows = [{"step": s, "validation_ce": ce} for s, ce in
            [(1000, 3.0), (2000, 2.5), (3000, 2.2), (4000, 2.1), (5000, 2.15)]]
    r = select_checkpoints(rows, targets=[2.5, 2.12, 1.5], tolerance=0.03)
    assert r["best_validation"] == {"step": 4000, "validation_ce": 2.1}
    assert r["iso_ce"]["2.5"]["step"] == 2000 and r["iso_ce"]["2.5"]["status"] == "matched"
    assert r["iso_ce"]["2.12"]["step"] == 4000 and r["iso_ce"]["2.12"]["target_reached"]
    far = r["iso_ce"]["1.5"]
    assert far["status"] == "outside_tolerance" and not far["target_reached"]
    assert select_checkpoints([], [2.0], 0.1) == {"best_validation": None, "iso_ce": {}}


def test_convergence_step_rule():
    rows = [{"step": s, "validation_ce": 3.0 * 0.9 ** (s // 5000) if s < 20000 else 2.18} for s in
            range(0, 40001, 5000)]
    # 15k -> 20k improves 0.3%: converged at 20k
    assert convergence_step(rows) == 20000
    assert convergence_step(rows[:3]) is None


def test_evaluate_checkpoints_scores_every_step(tmp_path, capsys):
    import torch
    from sigma0_b200.cli.train import main
    from sigma0_b200.data import LobWindowDataset, collate, make_sequences
    from sigma0_b200.models import preset_args
    from sigma0_b200.train.checkpoint_selection import evaluate_checkpoints
    from sigma0_b200.train.trainer import Trainer
    base = ["--preset", "smoke", "--impl", "torch", "--n_messages", "4", "--micro_bsz", "2", "--log_every", "1",
            "--watchdog_timeout", "0", "--synthetic", "2", "--no_validation", "--ckpt_dir", str(tmp_path / "ck")]
    assert main(base + ["--steps", "2", "--save_every", "1"]) == 0
    args = preset_args("smoke", impl="torch", n_messages=4, micro_bsz=2)
    days = make_sequences(2, 5, seed=9)
    ds = LobWindowDataset.from_days(days, 4, token_mode=args.token_mode)
    rows = evaluate_checkpoints(str(tmp_path / "ck"),
                                lambda: Trainer(args, device=torch.device("cpu"), total_steps=10),
                                lambda: [collate([ds[0], ds[1]])])
    assert [r["step"] for r in rows] == [1, 2] and all(np.isfinite(r["validation_ce"]) for r in rows)


def test_fidelity_real_arm_is_exact_and_a_corrupted_stream_diverges():
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.sim.fidelity import compare_paths, describe_stream, replay_stream, window_report
    d = make_sequences(1, 401, seed=3)[0]
    # the preprocessed layout holds the book BEFORE each message: the book after message i is row i + 1
    after = np.asarray(d.books[1:, 3:], np.int64)
    msgs = d.engine_msgs[:-1]
    init = np.asarray(d.l2_init, np.int64)
    real = window_report(init, msgs, after)["real"]
    assert real["clean"] and real["n_messages"] == 400
    assert real["exact_full_frac"] == 1.0 and real["first_divergence"] == -1
    # drop one new limit order from the middle of the stream: the path diverges from there on
    k = int(np.nonzero(msgs[:, 0] == 1)[0][len(msgs) // 8])
    path, _ = replay_stream(np.delete(msgs, k, 0), init)
    cmp = compare_paths(path, np.delete(after, k, 0))
    assert cmp["exact_full_frac"] < 1.0 and cmp["first_divergence"] >= 0
    m = msgs
    # a cancel naming an order nobody created is reported
    ghost = m.copy()
    ghost[5] = [3, 1, 10, ghost[5, 3], 123_456_789, 0, ghost[5, 6], ghost[5, 7]]
    r = describe_stream(ghost, prior_ids=[])
    assert r.n_unresolvable_ids >= 1 and r.n_unresolved_positive >= 1


def test_autopsy_finds_the_first_divergence_and_its_signature(tmp_path):
    """A stream replayed against its own books never diverges; against books recorded for a
    stream whose step k placed its order one tick away, the first divergence is step k, both
    books moved at disjoint prices, and the run-directory reader gives the same answer."""
    import pandas as pd
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.sim import divergence as A
    from sigma0_b200.sim.fidelity import replay_stream
    d = make_sequences(1, 301, seed=5)[0]
    after = np.asarray(d.books[1:, 3:], np.int64)
    msgs = np.asarray(d.engine_msgs[:-1], np.int64)
    init = np.asarray(d.l2_init, np.int64)
    assert A.first_divergence(msgs, after, init)["first_step"] == -1
    # the recorded books come from a stream whose k-th new order sat one tick deeper
    news = np.nonzero(msgs[:, 0] == 1)[0]
    # a new order that lands in the top three levels (deeper ones can fall off the compared book)
    top = lambda i: set(after[i].reshape(-1, 4)[:3, [0, 2]].reshape(-1).tolist())
    k = int(next(i for i in news[len(news) // 3:] if int(msgs[i, 3]) in top(i)))
    moved = msgs.copy()
    moved[k, 3] -= 100 * int(moved[k, 1])                 # a bid one tick lower, an ask one tick higher
    ref, _ = replay_stream(moved, init, after.shape[1] // 4)
    res = A.first_divergence(msgs, ref, init)
    assert res["first_step"] == k and res["message"]["type_name"] == "NEW"
    assert "DIFFERENT_PRICE" in res["signatures"] or "DIFFERENT_AMOUNT" in res["signatures"]
    # the same window written in the generation runtime's CSV layout
    for sub in ("data_cond", "data_gen"):
        (tmp_path / sub).mkdir()
    p = A.run_paths(str(tmp_path), "SYN", "2000-01-01", 7)
    pd.DataFrame(np.stack([init, init])).to_csv(p["cond_book"], index=False)
    pd.DataFrame({"time": [f"{s}.{ns:09d}" for s, ns in msgs[:, 6:8]], "event_type": msgs[:, 0],
                  "order_id": msgs[:, 4], "size": msgs[:, 2], "price": msgs[:, 3],
                  "direction": msgs[:, 1]}).to_csv(p["gen_msg"], index=False)
    pd.DataFrame(ref).to_csv(p["gen_book"], index=False)
    back = A.read_messages(p["gen_msg"])
    assert np.array_equal(back[:, [0, 1, 2, 3, 4, 6, 7]], msgs[:, [0, 1, 2, 3, 4, 6, 7]])
    w = A.autopsy_window(str(tmp_path), "SYN", "2000-01-01", 7)
    assert w["first_step"] == k and w["signatures"] == res["signatures"]
    assert A.autopsy_window(str(tmp_path), "SYN", "2000-01-01", 8) is None
    assert A.signatures(np.array([4, 1, 1, 1, -999_999_999, 0, 0, 0]), {}, {("bid", 1): 1}, 10) == \
        ["RECORDED_NOT_APPLIED", "AGGRESSIVE_EXECUTION", "MISS_SENTINEL"]
