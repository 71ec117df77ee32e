"""The training CLI's reference-compatible flags, validation, trace window and restore
options on CPU (``sigma0_b200/cli/train.py``)."""
import json
import os

import numpy as np
import pytest
import torch

# every flag of the reference's training runtime (run/base_model/runtime/train.py:47-330)
REFERENCE_TRAIN_FLAGS = """C_init USE_WANDB activation_fn attention_max_cache_len batchnorm bidirectional block_counts
block_size blocks bn_momentum book_ablation book_depth book_transform checkpoint_every_n_steps clip_eigs conj_sym
cosine_anneal curtail_epochs d_ff d_model data_root dataset debug_loading debug_overfit diloco_outer diloco_outer_lr
diloco_outer_momentum dir_name discretization dt_global dt_max dt_min dtype early_stop_patience enable_profiler epochs
gdn_chunk_size gdn_expand_v gdn_head_dim gdn_num_heads gdn_use_conv grad_accum_steps hierarchical hierarchical_nobook
hybrid_attn_d_ff hybrid_attn_flash hybrid_attn_heads hybrid_attn_layers hybrid_attn_positional_encoding ignore_times
jax_seed local_steps_k log_ce_tables lr_factor lr_min lr_patience mamba3_chunk_size mamba3_d_state mamba3_expand
mamba3_headdim mamba3_rope_fraction mamba3_use_cuda mamba3_use_triton masking max_grad_norm max_job_hours
max_train_batches merging micro_bsz mini_epochs mode model_type msg_seq_len muon_lr muon_wd n_book_post_layers
n_book_pre_layers n_data_workers n_heads n_layers n_message_layers no_validation num_devices opt_config p_dropout
partial_restore pe_type prefetch_factor prenorm random_offsets_train reduce_factor remat restore
restore_reset_schedule restore_step resume_from_step rope_base save_before_timeout_minutes shuffle_train
skip_test_eval ssm_lr_base ssm_size_base ssm_type test_date_range test_dir_name tickers token_mode tp_size
train_date_range uniform_ticker_batches use_book_data use_flash use_simple_book val_split wandb_entity wandb_project
warmup_end weight_decay window_size""".split()

BASE = ["--preset", "smoke", "--impl", "torch", "--n_messages", "4", "--micro_bsz", "2", "--log_every", "1",
        "--watchdog_timeout", "0"]


def _events(capsys):
    return [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]


def test_every_reference_training_flag_is_accepted():
    from sigma0_b200.cli.train import build_parser, parse
    opts = {o.lstrip("-") for act in build_parser()._actions for o in act.option_strings}
    assert not [f for f in REFERENCE_TRAIN_FLAGS if f not in opts]
    a = parse([])
    assert a.hierarchical is True and a.shuffle_train is True
    b = parse(["--use_book_data", "false", "--hierarchical", "False", "--checkpoint_every_n_steps", "auto"])
    assert b.use_book_data is False and b.hierarchical is False and b.save_every == "auto"


def test_reference_model_flags_reach_the_model_namespace():
    from sigma0_b200.cli.common import model_args
    from sigma0_b200.cli.train import _ref_model_extra, parse
    a = parse(BASE + ["--mamba3_d_state", "32", "--remat", "true", "--cosine_anneal", "false",
                      "--grad_accum_steps", "2", "--tp_size", "1", "--jax_seed", "5", "--msg_seq_len", "6"])
    args = model_args(a, **_ref_model_extra(a))
    assert args.mamba3_d_state == 32 and args.remat is True and args.cosine_anneal is False
    assert a.accum_steps == 2 and a.seed == 5 and a.n_messages == 6


def test_validation_early_stop_and_trace_window(tmp_path, capsys):
    from sigma0_b200.cli.train import main
    rc = main(BASE + ["--synthetic", "8", "--steps", "6", "--val_split", "0.25", "--eval_every", "1",
                      "--early_stop_patience", "1", "--lr", "0", "--lr_factor", "1",
                      "--profile_steps", "0,1", "--profile_dir", str(tmp_path / "prof")])
    assert rc == 0
    ev = _events(capsys)
    vals = [e for e in ev if "val_loss" in e]
    assert len(vals) >= 2 and all(v["val_loss"] == pytest.approx(vals[0]["val_loss"], rel=1e-6) for v in vals)
    fin = ev[-1]
    assert fin["stopped"] == "early_stop" and fin["steps"] == 2
    assert os.path.exists(tmp_path / "prof" / "trace_rank0.json")
    with open(tmp_path / "prof" / "trace_rank0.json") as f:
        assert "traceEvents" in json.load(f)


def test_reduce_on_plateau_lowers_the_lr_multiple():
    from sigma0_b200.train.loop import _Plateau

    class T:
        lr_mult = 1.0
    t = T()
    pl = _Plateau(early_stop_patience=0, lr_patience=2, reduce_factor=0.5)
    for v in (1.0, 1.1, 1.2, 1.3, 1.4):
        assert not pl.update(v, t)
    assert t.lr_mult == pytest.approx(0.25)
    pl.update(0.5, t)
    assert pl.best == 0.5


def test_remat_matches_the_plain_backward():
    from sigma0_b200.models import preset_args
    from sigma0_b200.models.registry import build_model
    torch.manual_seed(0)
    grads = []
    for remat in (False, True):
        args = preset_args("smoke", impl="torch", remat=remat, p_dropout=0.0)
        torch.manual_seed(0)
        m = build_model(args)
        tok = torch.randint(0, args.vocab_size, (2, 4 * args.msg_len))
        book = torch.randn(2, 4, args.d_book if hasattr(args, "d_book") else 503)
        loss, _ = m.loss(tok, book, tok)
        loss.backward()
        grads.append(torch.cat([p.grad.reshape(-1) for p in m.parameters() if p.grad is not None]))
    torch.testing.assert_close(grads[0], grads[1], rtol=1e-5, atol=1e-6)


def test_batchnorm_layers_train_and_keep_running_stats():
    from sigma0_b200.models import preset_args
    from sigma0_b200.models.common import BatchNorm
    from sigma0_b200.models.registry import build_model
    args = preset_args("smoke", impl="torch", batchnorm=True, bn_momentum=0.5)
    m = build_model(args)
    bns = [x for x in m.modules() if isinstance(x, BatchNorm)]
    assert bns and all(b.momentum == 0.5 for b in bns)
    tok = torch.randint(0, args.vocab_size, (2, 4 * args.msg_len))
    loss, _ = m.loss(tok, torch.randn(2, 4, 503), tok)
    loss.backward()
    assert torch.isfinite(loss) and bns[0].scale.grad is not None
    assert not torch.allclose(bns[0].mean, torch.zeros_like(bns[0].mean))
    m.eval()
    with torch.no_grad():
        l2, _ = m.loss(tok, torch.randn(2, 4, 503), tok)
    assert torch.isfinite(l2)


def test_partial_restore_from_another_run(tmp_path, capsys):
    from sigma0_b200.cli.train import main
    a = BASE + ["--synthetic", "2", "--no_validation"]
    assert main(a + ["--steps", "2", "--ckpt_dir", str(tmp_path / "one")]) == 0
    capsys.readouterr()
    assert main(a + ["--steps", "1", "--ckpt_dir", str(tmp_path / "two"), "--restore", str(tmp_path / "one"),
                     "--partial_restore"]) == 0
    ev = _events(capsys)
    r = [e for e in ev if e.get("event") == "restored"]
    assert r and r[0]["step"] == 2 and r[0]["params_only"] is True and r[0]["trainer_step"] == 0
    assert ev[-1]["steps"] == 1


def test_epochs_and_debug_overfit(capsys):
    from sigma0_b200.cli.train import main
    assert main(BASE + ["--synthetic", "4", "--epochs", "2", "--no_validation", "--debug_overfit", "true"]) == 0
    ev = _events(capsys)
    steps = [e for e in ev if "loss" in e and "step" in e]
    assert ev[-1]["steps"] == 4 and len(steps) == 4          # 2 epochs x 2 batches of 2 windows


def test_rl_runtime_reads_the_reference_ippo_keys(tmp_path):
    """``cli rl`` builds market makers and an executor on shared books from the reference's
    IPPO config keys and agent config field names, trains, and writes the policies."""
    import json
    from sigma0_b200.cli import rl
    cfg = {"NUM_ENVS": 2, "NUM_STEPS": 6, "TOTAL_TIMESTEPS": 24, "UPDATE_EPOCHS": 1, "NUM_MINIBATCHES": 2,
           "GAMMA": 0.99, "GAE_LAMBDA": 0.95, "CLIP_EPS": 0.2, "ENT_COEF": 0.01, "VF_COEF": 0.5,
           "GRU_HIDDEN_DIM": 16, "SEED": 3, "LR": [3e-4, 1e-4], "MAX_GRAD_NORM": [0.5, 1.0],
           "ANNEAL_LR": [True, False], "NUM_AGENTS_PER_TYPE": [2, 1], "MSGS_PER_STEP": 4, "WANDB_MODE": "off",
           "AGENT_CONFIGS": {"MarketMaking": {"action_space": "spread_skew", "reward_function": "spooner_damped",
                                              "inv_penalty": "quadratic", "unwind_price": "mid"},
                             "Execution": {"action_space": "fixed_quants_complex", "task": "random",
                                           "task_size": 200, "reward_function": "normal"}}}
    path = tmp_path / "ippo.json"
    path.write_text(json.dumps(cfg))
    assert rl.main(["--config", str(path), "--synthetic", "2", "--out", str(tmp_path / "out")]) == 0
    rec = json.loads((tmp_path / "out" / "history.json").read_text())
    assert rec["agent_types"] == ["mm", "exe"] and rec["iterations"] == 2 and rec["unused_config"] == ["WANDB_MODE"]
    assert (tmp_path / "out" / "policy_mm.pt").exists() and (tmp_path / "out" / "policy_exe.pt").exists()


def test_rl_runtime_fixed_time_episodes(tmp_path):
    """``world_config: {ep_type: fixed_time, episode_time}`` cuts the days into time windows and
    trains on environments whose episodes differ in length."""
    import json
    from sigma0_b200.cli import rl
    cfg = {"NUM_ENVS": 3, "NUM_STEPS": 4, "TOTAL_TIMESTEPS": 24, "UPDATE_EPOCHS": 1, "NUM_MINIBATCHES": 3,
           "GRU_HIDDEN_DIM": 8, "SEED": 1, "NUM_AGENTS_PER_TYPE": [1, 0], "MSGS_PER_STEP": 4,
           "world_config": {"ep_type": "fixed_time", "episode_time": 1, "last_step_seconds": 0}}
    assert rl.episode_config(cfg) == {"ep_type": "fixed_time", "episode_time": 1.0, "last_step_seconds": 0.0}
    assert rl.episode_config({}) == {"ep_type": "fixed_steps"}
    path = tmp_path / "ippo.json"
    path.write_text(json.dumps(cfg))
    assert rl.main(["--config", str(path), "--synthetic", "2", "--out", str(tmp_path / "out")]) == 0
    rec = json.loads((tmp_path / "out" / "history.json").read_text())
    assert rec["unused_config"] == [] and rec["history"]


def test_rl_baseline_only_sweeps_fixed_action_combinations(tmp_path):
    """``cli rl --baseline_only``: every combination of the per-type fixed actions, one row
    each with per-type returns, to JSON and CSV."""
    import json
    from sigma0_b200.cli import rl
    cfg = {"NUM_ENVS": 2, "NUM_STEPS": 5, "SEED": 2, "NUM_AGENTS_PER_TYPE": [1, 1], "MSGS_PER_STEP": 4,
           "AGENT_CONFIGS": {"MarketMaking": {}, "Execution": {"action_space": "fixed_quants_complex",
                                                               "task_size": 100}},
           "FIXED_ACTIONS": [[[0, 0], [1, 1], [2, 2]], [0, 4]]}
    path = tmp_path / "b.json"
    path.write_text(json.dumps(cfg))
    out = tmp_path / "out"
    assert rl.main(["--config", str(path), "--synthetic", "2", "--out", str(out), "--baseline_only"]) == 0
    rec = json.loads((out / "baselines.json").read_text())
    assert rec["agent_types"] == ["mm", "exe"] and len(rec["rows"]) == 6
    assert {tuple(r["mm_action"]) for r in rec["rows"]} == {(0, 0), (1, 1), (2, 2)}
    assert all(np.isfinite(r["mm_return"]) and np.isfinite(r["exe_return"]) for r in rec["rows"])
    assert (out / "baselines.csv").read_text().count("\n") == 7
    cfg["FIXED_ACTIONS"] = [[[0, 99]], [0]]
    path.write_text(json.dumps(cfg))
    with pytest.raises(ValueError, match="does not fit"):
        rl.main(["--config", str(path), "--synthetic", "2", "--out", str(out), "--baseline_only"])
