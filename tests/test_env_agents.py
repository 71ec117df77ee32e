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
                                    "twap": 1}[space], (3,), generator=rng)
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
