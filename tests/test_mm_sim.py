"""Closed-loop market-making simulator: replay and generator worlds (CPU)."""
import numpy as np
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
