"""Closed-loop market-making simulator: replay and generator worlds (CPU)."""
import numpy as np
import pytest
import torch

from sigma0_b200.data.synthetic import make_sequences
from sigma0_b200.encoding import get_tokenizer
from sigma0_b200.envs.baselines import fixed_offset
from sigma0_b200.sim import autopsy, build_episodes, run_episodes


def _episodes():
    return build_episodes(make_sequences(2, 40, seed=8), get_tokenizer("22tok"), n_ctx=6, n_future=20)


def test_replay_world():
    res = run_episodes(fixed_offset(0, 0), _episodes(), world="replay", steps=8, msgs_per_step=2)
    a = autopsy(res)
    assert res.steps == 8 and np.isfinite(a["pnl_ticks_mean"])
    assert abs(a["spread_capture_ticks_mean"] + a["inventory_pnl_ticks_mean"] - a["pnl_ticks_mean"]) < 1e-9


def test_generator_world_runs_with_agent_in_the_book():
    from sigma0_b200.models import preset_args, build_model
    torch.manual_seed(0)
    model = build_model(preset_args("smoke")).eval()
    res = run_episodes(fixed_offset(0, 0), _episodes(), world="generator", model=model, steps=3, msgs_per_step=2)
    assert res.steps == 3 and np.isfinite(res.pnl_ticks).all()


def test_frozen_episodes_signal_curve_and_the_replay_gate(tmp_path):
    """A frozen episode round-trips through its file and is never overwritten; a stream
    whose clock runs backwards is refused; the signal curve summarises rollouts per
    horizon; the replay gate of a run whose books come from the engine itself is exact."""
    import numpy as np
    import pandas as pd
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.sim import frozen as F
    from sigma0_b200.sim.divergence import run_paths
    from sigma0_b200.sim.fidelity import replay_stream
    d = make_sequences(1, 201, seed=2)[0]
    msgs = np.asarray(d.engine_msgs[:-1], np.int64)
    init = np.asarray(d.l2_init, np.int64)
    rollouts = [replay_stream(msgs[s:s + 50], init)[0] for s in (0, 50, 100)]
    sig = F.signal_curve(rollouts, [1, 10, 50, 80])
    assert sig["n_rollouts"] == 3 and np.isnan(sig["mid_mean"][3]) and \
        (sig["mid_q10"][:3] <= sig["mid_mean"][:3]).all() and (sig["mid_mean"][:3] <= sig["mid_q90"][:3]).all()
    spec = F.EpisodeSpec(12, "SYN", "2000-01-01", 7, (1, 2, 3), "bg-flow", "signal")
    ep = F.build_episode(spec, init, msgs, sig)
    path = F.save_episode(ep, str(tmp_path / "eps"))
    back = F.load_episode(path)
    assert np.array_equal(back["background"], msgs) and back["bg_checkpoint"] == "bg-flow"
    assert back["background_timing"]["monotonic"] and back["signal_seeds"].tolist() == [1, 2, 3]
    ep2 = dict(ep, background=msgs[:10])
    assert F.save_episode(ep2, str(tmp_path / "eps")) == path and \
        len(F.load_episode(path)["background"]) == len(msgs)            # the first file stays
    bad = msgs.copy()
    bad[20, 6] -= 5
    with pytest.raises(F.EpisodeError):
        F.build_episode(spec, init, bad, sig)
    # a run directory in the generation runtime's layout, its books from the engine itself
    for sub in ("data_cond", "data_gen"):
        (tmp_path / "run" / sub).mkdir(parents=True)
    root = str(tmp_path / "run")
    for i in (3, 9):
        p = run_paths(root, "SYN", "2000-01-01", i)
        m = msgs[20 * i:20 * i + 40]
        pd.DataFrame(np.stack([init])).to_csv(p["cond_book"], index=False)
        pd.DataFrame({"time": [f"{s}.{ns:09d}" for s, ns in m[:, 6:8]], "event_type": m[:, 0], "order_id": m[:, 4],
                      "size": m[:, 2], "price": m[:, 3], "direction": m[:, 1]}).to_csv(p["gen_msg"], index=False)
        pd.DataFrame(replay_stream(m, init)[0]).to_csv(p["gen_book"], index=False)
    assert F.run_windows(root, "SYN", 10) == [("2000-01-01", 3), ("2000-01-01", 9)]
    gate = F.replay_gate(root, "SYN")
    assert all(r["exact_mid_frac"] == 1.0 for r in gate.values()) and len(gate) == 2


def test_closed_loop_policy_against_a_frozen_episode():
    """The touch-quoting baseline trades against the background flow with exact accounting;
    a policy that never quotes ends flat at zero; one that raises ends its episode with an
    error; the inventory cap holds."""
    from sigma0_b200.sim import closed_loop as C
    from sigma0_b200.sim import frozen as F
    from sigma0_b200.data.synthetic import make_sequences
    d = make_sequences(1, 1500, seed=4)[0]
    msgs = np.asarray(d.engine_msgs[:-1], np.int64)
    ep = F.build_episode(F.EpisodeSpec(1, "SYN", "2000-01-01", 0, (0,)), np.asarray(d.l2_init, np.int64), msgs,
                         {"mid_mean": np.array([1.0, 2.0])})
    cfg = C.SimConfig(n_steps=30, warmup_s=0.0, size_cap=50, inventory_cap=120)
    t = C.run_frozen_episode(C.symmetric_touch, ep, cfg)
    assert t.error is None and t.n_fills > 0 and len(t.steps) > 0
    assert all(abs(s.inventory) <= cfg.inventory_cap + cfg.size_cap for s in t.steps)
    inv = sum((f["qty"] if f["side"] > 0 else -f["qty"]) for s in t.steps for f in s.fills)
    cash = -sum((f["qty"] if f["side"] > 0 else -f["qty"]) * f["px"] for s in t.steps for f in s.fills)
    assert inv == t.final_inventory and abs(cash - t.steps[-1].cash) < 1e-6
    assert abs(t.total_pnl - (t.realized_pnl + t.unwind_pnl)) < 1e-6
    idle = C.run_frozen_episode(lambda o, s: {}, ep, cfg)
    assert idle.n_fills == 0 and idle.total_pnl == 0.0
    seen = {}
    C.run_frozen_episode(lambda o, s: seen.setdefault("sig", o["signal"]) and {}, ep, cfg)
    assert seen["sig"]["mid_mean"] == [1.0, 2.0]

    def bad(o, s):
        raise RuntimeError("boom")
    err = C.run_frozen_episode(bad, ep, cfg)
    assert err.error and "boom" in err.error
    cmp = C.compare_to_baseline(C.symmetric_touch, [ep], cfg)
    assert cmp["delta_mean"] == 0.0 and not cmp["errors"]
