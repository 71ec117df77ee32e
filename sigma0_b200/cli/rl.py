"""Reinforcement-learning runtime: IPPO agents in the LOB environments.

``python -m sigma0_b200.cli rl --config ippo.yaml --synthetic 8 --out runs/rl``

The config is a YAML or JSON mapping with the reference's IPPO keys
(``environment/jaxrl/MARL/ippo_rnn_JAXMARL.py``, loaded there through hydra):

``NUM_ENVS``, ``NUM_STEPS`` (environment steps per episode), ``TOTAL_TIMESTEPS``,
``UPDATE_EPOCHS``, ``NUM_MINIBATCHES``, ``GAMMA``, ``GAE_LAMBDA``, ``CLIP_EPS``,
``ENT_COEF``, ``VF_COEF``, ``GRU_HIDDEN_DIM``, ``SEED``, per agent type (a list in
``NUM_AGENTS_PER_TYPE`` order, or one value for all) ``LR``, ``MAX_GRAD_NORM``,
``ANNEAL_LR``; ``NUM_AGENTS_PER_TYPE`` = [market makers, executors]; ``AGENT_CONFIGS``
with a ``MarketMaking`` and an ``Execution`` block in the reference's environment
config field names; ``MSGS_PER_STEP`` (data messages per environment step);
``world_config`` with ``ep_type`` (``fixed_steps``, or ``fixed_time`` windows of
``episode_time`` seconds) and ``last_step_seconds``.  Keys this
runtime does not use (logging, sweeps) are listed in the run record.

Data: ``--data_dir`` (preprocessed ``*_message.npy`` / ``*_book.npy`` day files) or
``--synthetic N`` seeded synthetic days.
Output under ``--out``: ``history.json`` (per-iteration returns and losses) and
``policy_<type>.pt`` (the actor-critics' state dicts).
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Dict, List

import torch

USED = {"NUM_ENVS", "NUM_STEPS", "TOTAL_TIMESTEPS", "UPDATE_EPOCHS", "NUM_MINIBATCHES", "GAMMA", "GAE_LAMBDA",
        "CLIP_EPS", "ENT_COEF", "VF_COEF", "GRU_HIDDEN_DIM", "SEED", "LR", "MAX_GRAD_NORM", "ANNEAL_LR",
        "NUM_AGENTS_PER_TYPE", "AGENT_CONFIGS", "MSGS_PER_STEP", "AUTOREGRESSIVE", "world_config", "WORLD_CONFIG",
        "EP_TYPE", "EPISODE_TIME", "LAST_STEP_SECONDS", "FIXED_ACTIONS"}

EXEC_CONFIG = {"action_space": "exec_action_space", "reward_function": "exec_reward", "task": "exec_task",
               "task_size": "exec_target", "fixed_quant_value": "exec_clip", "reward_lambda": "exec_lam"}


def load_config(path: str) -> Dict:
    with open(path) as f:
        text = f.read()
    if path.endswith(".json"):
        return json.loads(text)
    import yaml
    return yaml.safe_load(text) or {}


def _per_type(v, i: int):
    return v[i] if isinstance(v, (list, tuple)) else v


def episode_config(cfg: Dict) -> Dict:
    """Episode keywords of the environments from the config's ``world_config`` section (the
    reference's ``jaxob_config.py:233-240`` / ``config_io.py:96``): ``ep_type``
    (``fixed_steps`` or ``fixed_time``), ``episode_time`` in seconds for fixed-time episodes
    and ``last_step_seconds``; upper-case top-level keys are accepted too."""
    world = dict(cfg.get("world_config", {}) or cfg.get("WORLD_CONFIG", {}) or {})
    ep_type = world.get("ep_type", cfg.get("EP_TYPE", "fixed_steps"))
    out = {"ep_type": ep_type}
    if ep_type == "fixed_time":
        out["episode_time"] = float(world.get("episode_time", cfg.get("EPISODE_TIME", 1800)))
        lss = world.get("last_step_seconds", cfg.get("LAST_STEP_SECONDS"))
        if lss is not None:
            out["last_step_seconds"] = float(lss)
    return out


def build_env(cfg: Dict, windows, device: str = "cpu"):
    """The environment the config describes: market makers only, an executor only, or both
    on the same books."""
    from ..envs import ExecutionEnv, MarketMakingEnv, MultiAgentEnv
    n_mm, n_exec = (list(cfg.get("NUM_AGENTS_PER_TYPE", [1, 0])) + [0])[:2]
    agents = cfg.get("AGENT_CONFIGS", {}) or {}
    mm_cfg = dict(agents.get("MarketMaking", {}))
    ex_cfg = dict(agents.get("Execution", {}))
    common = dict(n_envs=int(cfg.get("NUM_ENVS", 8)), msgs_per_step=int(cfg.get("MSGS_PER_STEP", 5)),
                  seed=int(cfg.get("SEED", 0)), device=device, **episode_config(cfg))
    if n_mm == 0:
        kw = {"target": ex_cfg.pop("task_size", 500), "clip": ex_cfg.pop("fixed_quant_value", 10)}
        for k in ("action_space", "reward_function", "task", "reference_price"):
            if k in ex_cfg:
                kw[k] = ex_cfg.pop(k)
        if "reward_lambda" in ex_cfg:
            kw["lam"] = ex_cfg.pop("reward_lambda")
        if "doom_price_penalty" in ex_cfg:
            kw["doom_price_penalty"] = ex_cfg.pop("doom_price_penalty")
        return ExecutionEnv(windows, **common, **kw)
    if n_exec == 0:
        return MarketMakingEnv.from_reference_config(windows, common.pop("n_envs"), mm_cfg, n_mm=n_mm, **common)
    exec_kw = {EXEC_CONFIG[k]: v for k, v in ex_cfg.items() if k in EXEC_CONFIG}
    env = MultiAgentEnv.from_reference_config(windows, common.pop("n_envs"), mm_cfg, n_mm=n_mm, n_exec=n_exec,
                                              **exec_kw, **common)
    return env


def ppo_config(cfg: Dict, types: List[str]):
    from ..envs.ippo import PPOConfig
    per = {t: {"lr": float(_per_type(cfg.get("LR", 3e-4), i)),
               "max_grad_norm": float(_per_type(cfg.get("MAX_GRAD_NORM", 0.5), i)),
               "anneal_lr": bool(_per_type(cfg.get("ANNEAL_LR", False), i))} for i, t in enumerate(types)}
    return PPOConfig(gamma=float(cfg.get("GAMMA", 0.99)), lam=float(cfg.get("GAE_LAMBDA", 0.95)),
                     clip=float(cfg.get("CLIP_EPS", 0.2)), epochs=int(cfg.get("UPDATE_EPOCHS", 4)),
                     minibatches=int(cfg.get("NUM_MINIBATCHES", 1)), ent_coef=float(cfg.get("ENT_COEF", 0.01)),
                     vf_coef=float(cfg.get("VF_COEF", 0.5)), hidden=int(cfg.get("GRU_HIDDEN_DIM", 64)),
                     autoregressive=bool(cfg.get("AUTOREGRESSIVE", False)), per_type=per)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="sigma0-b200 IPPO runtime")
    p.add_argument("--config", required=True)
    p.add_argument("--data_dir", default=None)
    p.add_argument("--synthetic", type=int, default=0)
    p.add_argument("--out", required=True)
    p.add_argument("--device", default="cpu", help="engine device: cpu (oracle) or cuda (batched kernel)")
    p.add_argument("--baseline_only", action="store_true",
                   help="no training: every combination of the config's FIXED_ACTIONS per agent type, "
                        "written to baselines.json / baselines.csv")
    p.add_argument("--episodes", type=int, default=1, help="episodes per combination with --baseline_only")
    a = p.parse_args(argv)
    cfg = load_config(a.config)
    from ..envs import windows_from_days
    steps = int(cfg.get("NUM_STEPS", 20))
    mps = int(cfg.get("MSGS_PER_STEP", 5))
    from .common import load_days
    days = load_days(a.data_dir, max(1, a.synthetic or 4), steps * mps * 4 + 1, int(cfg.get("SEED", 0)))
    ep = episode_config(cfg)
    if ep["ep_type"] == "fixed_time":
        windows = windows_from_days(days, length=int(ep["episode_time"]), ep_type="fixed_time", msgs_per_step=mps)
    else:
        windows = windows_from_days(days, length=steps * mps)
    env = build_env(cfg, windows, a.device)
    from ..envs.ippo import _groups, train_ippo
    types = [g.name for g in _groups(env)]
    if a.baseline_only:
        return _baseline_only(cfg, env, types, a)
    iters = max(1, int(cfg.get("TOTAL_TIMESTEPS", steps * env.n)) // (steps * env.n))
    os.makedirs(a.out, exist_ok=True)
    hist, pol = train_ippo(env, iterations=iters, cfg=ppo_config(cfg, types), seed=int(cfg.get("SEED", 0)),
                           log=lambda r: print(json.dumps(r), flush=True))
    pols = pol if isinstance(pol, dict) else {types[0]: pol}
    for t, m in pols.items():
        torch.save(m.state_dict(), os.path.join(a.out, f"policy_{t}.pt"))
    with open(os.path.join(a.out, "history.json"), "w") as f:
        json.dump({"history": hist, "agent_types": types, "iterations": iters,
                   "unused_config": sorted(k for k in cfg if k not in USED)}, f, indent=1)
    return 0


def _baseline_only(cfg: Dict, env, types: List[str], a) -> int:
    """FIXED_ACTIONS: a list in agent-type order or a {type: ...} map; per type a list of the
    actions to try (each an int or one int per action dimension), or one bare int."""
    from ..envs.baselines import fixed_action_sweep
    fa = cfg.get("FIXED_ACTIONS")
    if fa is None:
        raise ValueError("--baseline_only needs FIXED_ACTIONS in the config")
    per = fa if isinstance(fa, dict) else {t: fa[i] for i, t in enumerate(types) if i < len(fa)}
    per = {t: (v if isinstance(v, (list, tuple)) else [v]) for t, v in per.items()}
    rows = fixed_action_sweep(env, per, episodes=a.episodes)
    os.makedirs(a.out, exist_ok=True)
    with open(os.path.join(a.out, "baselines.json"), "w") as f:
        json.dump({"agent_types": types, "episodes": a.episodes, "rows": rows}, f, indent=1)
    import csv
    keys = list(rows[0])
    with open(os.path.join(a.out, "baselines.csv"), "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=keys)
        w.writeheader()
        for r in rows:
            w.writerow({k: (" ".join(map(str, v)) if isinstance(v, list) else v) for k, v in r.items()})
    for r in rows:
        print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
