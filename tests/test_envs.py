"""Environments on the batched engine: fills, market making baselines, execution, PPO."""
import numpy as np
import torch

from sigma0_b200.data.synthetic import make_sequences
from sigma0_b200.envs import MarketMakingEnv, ExecutionEnv, MultiAgentEnv, windows_from_days


def _windows():
    return windows_from_days(make_sequences(3, 120, seed=5), length=60)


def test_market_maker_fills_match_inventory_and_cash():
    env = MarketMakingEnv(_windows(), n_envs=4, msgs_per_step=5, seed=1)
    obs = env.reset()
    # tight quotes on both sides so the replayed flow trades against them
    tot_q = torch.zeros(4, 1, dtype=torch.long)
    while not env.done:
        obs, r, _ = env.step(torch.zeros(4, 1, 2, dtype=torch.long))
        assert torch.isfinite(r).all()
    assert env.inv.abs().sum() > 0 or env.cash.abs().sum() > 0        # some activity happened
    # PnL identity: cash + inventory * mid
    mid = env.observe()["mid"].double()
    assert torch.allclose(env.pnl_prev[:, 0], env.cash[:, 0] + env.inv[:, 0].double() * mid)


def test_crossing_quote_is_an_aggressor_fill():
    env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=1, seed=2)
    obs = env.reset()
    best_ask = obs["l2"][:, 0].clone()
    # a bid at the best ask crosses: emulate by offset below the mid that reaches the ask
    mid = obs["mid"]
    msgs = env.action_messages(torch.zeros(2, 1, 2, dtype=torch.long), mid)
    msgs[:, 2, 3] = best_ask                     # the new bid (row 2) at the best ask
    msgs[:, 3] = 0                               # no ask quote this step
    ask_vol = obs["l2"][:, 1].clone()
    trades, _ = env.step_messages(msgs)
    for b in range(2):
        first = trades[b, 0]                     # the agent's bid trades first, as aggressor
        assert first[0] == best_ask[b] and first[7] == env.tids[0]
        assert -first[1] == min(100, int(ask_vol[b]))


def test_baselines_and_execution():
    from sigma0_b200.envs.baselines import avellaneda_stoikov, fixed_offset, evaluate
    env = MarketMakingEnv(_windows(), n_envs=3, msgs_per_step=5, seed=3)
    a = evaluate(env, avellaneda_stoikov())
    b = evaluate(env, fixed_offset(0, 0))
    assert np.isfinite(a["pnl_ticks_mean"]) and np.isfinite(b["pnl_ticks_mean"])
    ex = ExecutionEnv(_windows(), n_envs=3, msgs_per_step=5, target=300, seed=4)
    o = ex.reset()
    while not ex.done:
        o, r, _ = ex.step(torch.full((3,), 2, dtype=torch.long))
    assert (ex.done_qty > 0).all() and (ex.done_qty <= 300).all()


def test_multi_agent_and_ppo():
    from sigma0_b200.envs.ippo import train_ippo, PPOConfig
    env = MultiAgentEnv(_windows(), n_envs=3, msgs_per_step=5, n_mm=2, seed=6)
    env.reset()
    o, r, _ = env.step(torch.zeros(3, 2, 2, dtype=torch.long), exec_qty=torch.full((3,), 50))
    assert r.shape == (3, 2)
    hist, pol = train_ippo(MarketMakingEnv(_windows(), n_envs=4, msgs_per_step=6, seed=7), iterations=2,
                           cfg=PPOConfig(epochs=2))
    assert len(hist) == 2 and all(np.isfinite(h["loss"]) for h in hist)


def test_market_makers_and_executors_share_the_books():
    """Two market makers and two executors (one buying, one selling at random per env) on the
    same books: cancels go first, rewards come per agent, the executors finish their task."""
    env = MultiAgentEnv(_windows(), n_envs=3, msgs_per_step=5, n_mm=2, n_exec=2, seed=8, exec_target=300,
                        exec_task="random", exec_action_space="fixed_quants_complex", exec_reward="normal",
                        action_space="spread_skew", reward_function="spooner", shuffle_action_messages=True)
    obs = env.reset()
    rng = torch.Generator().manual_seed(3)
    msgs = env._order(env.action_messages(torch.randint(0, 5, (3, 2, 2), generator=rng), obs["mid"]))
    typ = msgs[..., 0]
    first_new = (typ != 3).float().argmax(1)
    assert all(bool((typ[i, first_new[i]:] != 3).all()) for i in range(3))     # no cancel after a new order
    while not env.done:
        obs, rew, done = env.step(torch.randint(0, 5, (3, 2, 2), generator=rng),
                                  exec_actions=torch.randint(0, 13, (3, 2), generator=rng))
        assert rew.shape == (3, 4) and torch.isfinite(rew).all()
    assert (obs["exec_remaining"] <= 300).all() and (env.exec_done > 0).any()


def test_ippo_per_agent_type_with_multi_discrete_and_autoregressive_heads():
    """IPPO trains one actor-critic per agent type: two market makers on a two-dimensional
    action space (autoregressive heads) and an executor on the 13-action ladder share the
    books; an executor alone trains too."""
    from sigma0_b200.envs.ippo import PPOConfig, action_dims, train_ippo
    assert action_dims("mm", "spread_skew") == (5, 5) and action_dims("mm", "fixed_prices", 2) == (3,) * 4
    env = MultiAgentEnv(_windows(), n_envs=3, msgs_per_step=5, n_mm=2, n_exec=1, seed=4, exec_target=200,
                        exec_task="random", exec_action_space="fixed_quants_complex", exec_reward="normal",
                        action_space="spread_skew", reward_function="spooner")
    cfg = PPOConfig(epochs=2, minibatches=2, autoregressive=True, anneal_lr=True, per_type={"exe": {"lr": 1e-4}})
    hist, pols = train_ippo(env, iterations=2, cfg=cfg)
    assert set(pols) == {"mm", "exe"} and pols["mm"].dims == (5, 5) and pols["exe"].dims == (13,)
    assert all(np.isfinite(h["mm_loss"]) and np.isfinite(h["exe_loss"]) for h in hist)
    ex = ExecutionEnv(_windows(), n_envs=3, msgs_per_step=5, target=300, seed=4, action_space="fixed_prices")
    hist, pol = train_ippo(ex, iterations=1, cfg=PPOConfig(epochs=1))
    assert pol.dims == (3, 3, 3, 3) and np.isfinite(hist[0]["loss"])


def test_multiplicative_weights_bandit_baseline():
    from sigma0_b200.envs.baselines import MultiplicativeWeights, run_bandit
    b = MultiplicativeWeights(4, eta=0.5, n_envs=2, n_agents=1, seed=0)
    b.last = torch.tensor([[3], [0]])
    b.update(torch.tensor([[2.0], [-2.0]]))
    assert torch.allclose(b.w.sum(-1), torch.ones(2, 1, dtype=torch.float64))
    assert b.w[0, 0].argmax() == 3 and b.w[1, 0, 0] < b.w[1, 0, 1]
    env = MarketMakingEnv(_windows(), n_envs=3, msgs_per_step=5, seed=2, action_space="fixed_quants",
                          reward_function="spooner")
    res = run_bandit(env, MultiplicativeWeights(8, eta=0.05, n_envs=3, seed=1))
    assert np.isfinite(res["reward_mean"]) and 1 / 8 <= res["weights_max_mean"] <= 1


def _ippo_rank(rank, world, port, out):
    import os
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from sigma0_b200.envs.ippo import PPOConfig, train_ippo
        torch.set_num_threads(1)
        # each rank runs its own environments (different windows), the same initial policy
        env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=6, seed=10 + rank, action_space="bobRL")
        _, pol = train_ippo(env, iterations=2, cfg=PPOConfig(epochs=1), seed=0)
        flat = torch.cat([p.detach().reshape(-1) for p in pol.parameters()])
        allp = [torch.zeros_like(flat) for _ in range(world)]
        dist.all_gather(allp, flat)
        if rank == 0:
            torch.save({"same": all(torch.equal(allp[0], x) for x in allp)}, out)
    finally:
        dist.destroy_process_group()


def test_ippo_ranks_average_gradients_and_stay_identical(tmp_path):
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "r.pt")
    mp.spawn(_ippo_rank, args=(2, port, out), nprocs=2, join=True)
    assert torch.load(out)["same"]


def test_observation_flags_an_empty_book_side():
    env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=5, seed=1)
    obs = env.reset()
    assert not obs["abort_episode"].any()
    # wipe the bid side of env 0 with deletes of every resting bid
    asks, bids = env.engine.sides()
    rows = [[3, 1, int(q), int(p), int(oid), 0, 0, 0] for p, q, oid, *_ in bids[0] if q > 0]
    msgs = torch.zeros(2, len(rows), 8, dtype=torch.int32)
    msgs[0] = torch.tensor(rows, dtype=torch.int32)
    env.engine.process(msgs.numpy() if not env.engine.on_gpu else msgs)
    o = env.observe()
    assert bool(o["abort_episode"][0]) and not bool(o["abort_episode"][1])


def _timed_day(seed=3, n=600):
    """A synthetic day whose messages arrive at irregular times over about 30 seconds."""
    from types import SimpleNamespace
    d = make_sequences(1, n, seed=seed)[0]
    rng = np.random.default_rng(seed)
    t = np.cumsum(rng.exponential(0.05, size=n)) * (1 + 0.8 * np.sin(np.arange(n) / 40.0) ** 2)
    t = np.maximum.accumulate(t)
    msgs = d.engine_msgs.copy()
    msgs[:, 6] = 34200 + t.astype(np.int64)
    msgs[:, 7] = ((t % 1) * 1e9).astype(np.int64)
    books = d.books.copy()
    books[:, 1], books[:, 2] = msgs[:, 6], msgs[:, 7]
    return SimpleNamespace(engine_msgs=msgs, books=books)


def test_fixed_time_episodes():
    day = _timed_day()
    k = 5
    ws = windows_from_days([day], length=3, ep_type="fixed_time", msgs_per_step=k)
    lens = [w.engine_msgs.shape[0] for w in ws]
    assert len(set(lens)) > 1 and all(n % k == 0 and n > 0 for n in lens)
    for w in ws:                                   # one 3-second interval each
        sec = w.engine_msgs[:, 6]
        assert (sec - 34200) .min() // 3 == (sec - 34200).max() // 3
    order = np.argsort(lens)
    idx = [int(order[0]), int(order[-1]), int(order[len(order) // 2]), int(order[1])]
    env = MarketMakingEnv(ws, n_envs=4, msgs_per_step=k, seed=1, ep_type="fixed_time", episode_time=3,
                          unwind_price="mid", last_step_seconds=0.5)
    obs = env.reset(idx)
    steps = env.steps_env.clone()
    assert steps.tolist() == [lens[i] // k for i in idx]
    assert torch.all(obs["time_left"] <= 1.0)
    prev_tl = obs["time_left"].clone()
    n_steps, books_at_end = 0, {}
    while not env.done:
        obs, r, _ = env.step(torch.zeros(4, 1, 2, dtype=torch.long))
        n_steps += 1
        assert torch.all(obs["time_left"] <= prev_tl + 1e-6)
        prev_tl = obs["time_left"].clone()
        for e in range(4):
            if n_steps == int(steps[e]):
                books_at_end[e] = obs["l2"][e].clone()
                assert env.inv[e, 0] == 0                        # the unwind flattened it
            elif n_steps > int(steps[e]):
                assert r[e].abs().sum() == 0                     # frozen: no reward
                assert torch.equal(obs["l2"][e], books_at_end[e])  # and no book change
    assert n_steps == int(steps.max())
    # execution: TWAP spreads the target over each environment's own steps; the last step sweeps
    ex = ExecutionEnv(ws, n_envs=4, msgs_per_step=k, seed=1, ep_type="fixed_time", episode_time=3,
                      target=200, action_space="twap", task="buy", last_step_seconds=0.0)
    ex.reset(idx)
    while not ex.done:
        _, r, _ = ex.step(torch.zeros(4, dtype=torch.long))
    assert torch.all(ex.done_qty == 200) and torch.all(ex.info["quant_left"] == 0)
    try:
        MarketMakingEnv(ws, n_envs=2, ep_type="fixed_time")
    except ValueError as e:
        assert "episode_time" in str(e)
    else:
        raise AssertionError("fixed_time without episode_time accepted")
