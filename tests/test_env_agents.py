"""Action spaces and rewards of the market-making and execution agents
(``envs/agents.py`` on the batched engine, CPU)."""
import pytest
import torch

from sigma0_b200.envs import ExecutionEnv, MarketMakingEnv
from sigma0_b200.envs.agents import (EXEC_ACTION_SPACES, MM_ACTION_SPACES, MM_REWARDS, agent_trades, exec_reward,
                                     mm_orders, mm_reward)

from test_envs import _windows


def _action(space, n, rng):
    if space in ("offsets", "bobRL", "spread_skew"):
        hi = {"offsets": (5, 5), "bobRL": (5, 3), "spread_skew": (5, 5)}[space]
        return torch.stack([torch.randint(0, h, (n,), generator=rng) for h in hi], -1)
    if space == "fixed_prices":
        return torch.randint(0, 3, (n, 6), generator=rng)
    hi = {"fixed_quants": 8, "AvSt": 8, "bobStrategy": 5, "directional_trading": 5, "simple": 4}[space]
    return torch.randint(0, hi, (n,), generator=rng)


@pytest.mark.parametrize("space", MM_ACTION_SPACES)
def test_every_market_making_action_space_runs_an_episode(space):
    env = MarketMakingEnv(_windows(), n_envs=3, msgs_per_step=5, seed=11, action_space=space,
                          reward_function="spooner")
    env.reset()
    rng = torch.Generator().manual_seed(0)
    total = torch.zeros(3, 1, dtype=torch.float64)
    for _ in range(env.max_steps):
        obs, rew, done = env.step(_action(space, 3, rng)[:, None])
        assert torch.isfinite(rew).all()
        total += rew
    assert done


def test_directional_market_buy_fills_and_simple_none_quotes_nothing():
    env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=1, seed=2, action_space="directional_trading")
    env.reset()
    obs, _, _ = env.step(torch.ones(2, 1, dtype=torch.long))          # market buy
    assert (obs["inventory"][:, 0] > 0).all()
    env2 = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=1, seed=2, action_space="simple")
    env2.reset()
    msgs = env2.action_messages(torch.full((2, 1), 3, dtype=torch.long))
    assert int((msgs[..., 0] != 0).sum()) == 0                        # nothing to cancel, nothing quoted


def test_avellaneda_stoikov_quotes_lean_against_inventory():
    st = {"best_bid": torch.tensor([9900]), "best_ask": torch.tensor([10100]), "mid": torch.tensor([10000]),
          "time_left": torch.tensor([1.0])}
    flat, _ = mm_orders("AvSt", torch.tensor([3]), dict(st, inventory=torch.tensor([0])), 100, 100)
    long, _ = mm_orders("AvSt", torch.tensor([3]), dict(st, inventory=torch.tensor([300])), 100, 100)
    assert long[0, 0, 1] < flat[0, 0, 1] and long[0, 1, 1] < flat[0, 1, 1]     # both quotes lower when long
    assert flat[0, 0, 1] < 10000 < flat[0, 1, 1]


def test_reward_formulas():
    t = lambda *v: torch.tensor(v, dtype=torch.float64)
    kw = dict(buy_q=t(100), buy_v=t(100 * 9900), sell_q=t(0), sell_v=t(0), inv_prev=t(50), inv=t(150),
              cash=t(-100 * 9900), mid0=t(10000), mid1=t(10100), best_bid=t(10000), best_ask=t(10200), tick=100)
    bs = (10100 - 9900) * 100 / 100          # bought 100 two ticks under the (new) mid
    inv_pnl = 50 * 100 / 100                 # 50 held while the mid rose one tick
    assert float(mm_reward("buy_sell_pnl", **kw)[0]) == pytest.approx(bs)
    assert float(mm_reward("spooner", **kw)[0]) == pytest.approx(bs + inv_pnl)
    assert float(mm_reward("spooner_damped", eta=0.5, **kw)[0]) == pytest.approx(bs + 0.5 * inv_pnl)
    assert float(mm_reward("spooner_asym_damped", eta=0.5, **kw)[0]) == pytest.approx(bs + 0.5 * inv_pnl)
    assert float(mm_reward("zero_inv", **kw)[0]) == pytest.approx(-150)
    pv = -100 * 9900 / 100 + 150 * 10100 / 100
    assert float(mm_reward("portfolio_value", **kw)[0]) == pytest.approx(pv)
    assert float(mm_reward("complex", eta=0.5, lam=0.1, **kw)[0]) == pytest.approx(bs + 0.5 * inv_pnl - 0.1 * 100)
    assert set(MM_REWARDS) >= {"portfolio_value", "buy_sell_pnl", "complex", "zero_inv", "spooner",
                               "spooner_damped", "spooner_asym_damped", "spooner_asym_damped2", "spooner_scaled",
                               "delta_portfolio_value"}


@pytest.mark.parametrize("space", EXEC_ACTION_SPACES)
def test_every_execution_action_space_completes_the_target(space):
    env = ExecutionEnv(_windows(), n_envs=3, msgs_per_step=5, target=300, seed=4, action_space=space,
                       reward_function="vwap")
    env.reset()
    rng = torch.Generator().manual_seed(1)
    for _ in range(env.max_steps):
        if space == "fixed_prices":
            act = torch.randint(0, 2, (3, 4), generator=rng)
        else:
            act = torch.randint(0, {"sizes": 5, "fixed_quants": 6, "fixed_quants_1msg": 5, "simplest_case": 2,
                                    "twap": 1, "fixed_quants_complex": 13}[space], (3,), generator=rng)
        obs, rew, done = env.step(act)
        assert torch.isfinite(rew).all()
    assert done
    # the final sweep completes the task where the book has the liquidity
    assert (obs["remaining"] <= 0).any()


def test_vwap_reward_rewards_buying_below_the_market():
    t = lambda *v: torch.tensor(v)
    kw = dict(market_q=t(1000), market_v=t(1000 * 10050), arrival=t(10000), target=100, tick=100, lam=0.0)
    good = exec_reward("vwap", filled=t(100), value=t(100 * 10000), sell=False, **kw)
    bad = exec_reward("vwap", filled=t(100), value=t(100 * 10100), sell=False, **kw)
    assert float(good) > 0 > float(bad)
    sell_good = exec_reward("vwap", filled=t(100), value=t(100 * 10100), sell=True, **kw)
    assert float(sell_good) > 0


def test_agent_trades_splits_buys_and_sells():
    # rows: price, qty, ..., passive tid (6), aggressor tid (7); qty signed from the resting side:
    # the passive trader's fill is +qty, the aggressor's -qty
    tr = torch.zeros(1, 3, 8, dtype=torch.long)
    tr[0, 0] = torch.tensor([100, -5, 0, 0, 0, 0, 7, 9])    # tid 7's resting ask lifted: 7 sold 5 at 100
    tr[0, 1] = torch.tensor([101, -4, 0, 0, 0, 0, 3, 7])    # tid 7 lifted an ask: bought 4 at 101
    tr[0, 2] = -1
    bq, bv, sq, sv = agent_trades(tr, 7)
    assert (int(bq), int(bv), int(sq), int(sv)) == (4, 404, 5, 500)


def test_episode_end_unwind_flattens_the_inventory_at_the_unwind_price():
    """unwind_price: the last step adds one artificial fill of the remaining inventory at the
    chosen price, moved unwind_penalty ticks against the agent."""
    from sigma0_b200.envs.agents import unwind_fill
    t = lambda *v: torch.tensor(v, dtype=torch.long)
    bq, bv, sq, sv = unwind_fill("far_touch", t(300, -200, 0), t(10000, 10000, 10000), t(10100, 10100, 10100),
                                 t(10000, 10000, 10000), t(10200, 10200, 10200), 100, penalty_ticks=2)
    assert sq.tolist() == [300, 0, 0] and bq.tolist() == [0, 200, 0]
    assert sv[0] == 300 * (10000 - 200) and bv[1] == 200 * (10200 + 200)
    _, _, sq, sv = unwind_fill("mid_avg", t(10), t(10000), t(10200), t(0), t(0), 100)
    assert sv[0] == 10 * 10100
    env = MarketMakingEnv(_windows(), n_envs=3, msgs_per_step=5, seed=3, action_space="directional_trading",
                          reward_function="spooner", unwind_price="mid")
    env.reset()
    for k in range(env.max_steps):
        obs, rew, done = env.step(torch.ones(3, 1, dtype=torch.long) if k < 2 else torch.zeros(3, 1, dtype=torch.long))
        assert torch.isfinite(rew).all()
    assert done and (obs["inventory"] == 0).all() and (env.unwound[:, 0] > 0).all()


def test_auto_liquidation_replaces_the_quotes_by_an_order_against_the_position():
    env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=1, seed=2, action_space="fixed_quants",
                          auto_liquidate_threshold=50, auto_liquidate_alpha=0.5)
    env.reset()
    env.inv[:, 0] = torch.tensor([120, 10])
    msgs = env.action_messages(torch.zeros(2, 1, dtype=torch.long))
    new = msgs[..., 0] == 1
    assert int(new[0].sum()) == 0 and int(new[1].sum()) > 0          # env 0 quotes nothing
    mkt = msgs[0][msgs[0, :, 0] == 4]
    assert mkt.shape[0] == 1 and int(mkt[0, 2]) == 60 and int(mkt[0, 1]) == 1   # sell 60 against the bids
    assert int((msgs[1, :, 0] == 4).sum()) == 0


def test_reward_shaping_options_and_observation_spaces():
    from sigma0_b200.envs.agents import inventory_penalty
    q = torch.tensor([0, 500, 1500])
    assert inventory_penalty("threshold", q, 1.0, 100, threshold=10.0).tolist() == [0.0, 0.0, -225.0]
    assert inventory_penalty("exp4", torch.tensor([0]), 2.0, 100).tolist() == [-2.0]
    rng = torch.Generator().manual_seed(1)
    for kw in (dict(clip_reward=True), dict(volume_bonus="market_share"), dict(exclude_extreme_spreads=True)):
        env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=5, seed=4, action_space="spread_skew",
                              reward_function="spooner", **kw)
        env.reset()
        for _ in range(3):
            _, rew, _ = env.step(_action("spread_skew", 2, rng)[:, None])
            assert torch.isfinite(rew).all()
            if "clip_reward" in kw:
                assert rew.abs().max() <= 10000
    env = MarketMakingEnv(_windows(), n_envs=2, msgs_per_step=5, seed=4, observation_space="engineered")
    obs = env.reset()
    obs["inventory"][:, 0] = torch.tensor([20, -30])
    v = env.agent_observation(obs)
    assert v.shape == (2, 1, 2) and v[:, 0, 0].tolist() == [2.0, -3.0]
    assert torch.allclose(v[:, 0, 1].double(), (obs["spread"] * env.tick).double() / 1e4)
    env.obs_space = "basic"
    assert env.agent_observation(obs).shape == (2, 1, 1)
    env.obs_space = "messages"
    assert env.agent_observation(obs).shape == (2, 1, 40) and not env.agent_observation(obs).any()
    obs, _, _ = env.step(torch.zeros(2, 1, 2, dtype=torch.long))
    assert torch.equal(env.agent_observation(obs)[:, 0], env.data[:, :5].reshape(2, -1).float())


def test_market_maker_from_the_reference_config_names():
    cfg = {"action_space": "spread_skew", "reward_function": "spooner_asym_damped2", "inv_penalty": "threshold",
           "inv_penalty_lambda": 0.5, "inv_penalty_threshold": 3.0, "unwind_price": "far_touch",
           "unwind_price_penalty": 5, "reference_price": "mid_avg", "inventoryPnL_eta": 0.6,
           "inventoryPnL_gamma": 0.5, "rebate_bps": 10.0, "clip_reward": True, "debug_mode": False,
           "observation_space": "messages_new_tokenizer"}
    env = MarketMakingEnv.from_reference_config(_windows(), 2, cfg, msgs_per_step=5, seed=1)
    assert (env.space, env.reward_fn, env.inv_pen_kind, env.unwind, env.unwind_pen) == \
        ("spread_skew", "spooner_asym_damped2", "threshold", "far_touch", 5)
    assert env.pen == 0.5 and env.eta == 0.6 and env.clip and env.ref_price == "mid_avg"
    assert set(env.unused_config) == {"debug_mode", "observation_space"}
    env.reset()
    rng = torch.Generator().manual_seed(0)
    for _ in range(env.max_steps):
        _, rew, done = env.step(_action("spread_skew", 2, rng)[:, None])
        assert torch.isfinite(rew).all()
    assert done


def test_execution_random_tasks_unwind_and_the_reference_rewards():
    """task='random' draws a side per environment; end_fn='unwind' books what is left at the
    far touch moved doom_price_penalty ticks against the agent; the reference's rewards."""
    env = ExecutionEnv(_windows(), n_envs=8, msgs_per_step=5, target=400, seed=9, task="random",
                       action_space="fixed_quants_complex", reward_function="normal", end_fn="unwind",
                       reference_price="far_touch", doom_price_penalty=3)
    obs = env.reset()
    sells = obs["is_sell"].clone()
    for _ in range(env.max_steps):
        obs, rew, done = env.step(torch.zeros(8, dtype=torch.long))          # never trade
        assert torch.isfinite(rew).all()
    assert done and (obs["remaining"] == 0).all() and (env.info["doom_quant"] == 400).all()
    # sellers receive cash, buyers pay it
    assert ((env.cash > 0) == sells).all()
    t = lambda *v: torch.tensor(v, dtype=torch.float64)
    r = exec_reward("normal", filled=t(100), value=t(100 * 9900), market_q=t(50), market_v=t(50 * 10000),
                    arrival=t(10000), target=400, sell=False, tick=100, lam=0.0)
    assert float(r[0]) == 100.0                      # bought 1 tick below the VWAP, 100 shares
    r = exec_reward("finish_fast", filled=t(0), value=t(0), market_q=t(0), market_v=t(0), arrival=t(1),
                    target=1, sell=True, tick=100, remaining=torch.tensor([250]))
    assert float(r[0]) == -250.0
    r = exec_reward("simplest_case", filled=t(10), value=t(10 * 10100), market_q=t(0), market_v=t(0),
                    arrival=t(10000), target=1, sell=True, tick=100)
    assert float(r[0]) == 1000.0                     # sold 100 above the arrival price, 10 shares
