"""The environments on the batched CUDA engine (one warp per book) take exactly the steps
they take on the CPU oracle engine: same fills, inventories, cash and rewards."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _windows():
    from sigma0_b200.data import make_sequences
    from sigma0_b200.envs import windows_from_days
    return windows_from_days(make_sequences(3, 120, seed=5), length=60)


def _run(cls, device, steps_fn, **kw):
    env = cls(_windows(), device=device, **kw)
    env.reset(idx=[0, 1, 2, 0])
    out = []
    gen = torch.Generator().manual_seed(0)
    while not env.done:
        _, r, _ = steps_fn(env, gen)
        out.append(r.double().clone())
    return env, torch.stack(out)


def test_market_making_and_execution_envs_match_on_the_cuda_engine():
    from sigma0_b200.envs import ExecutionEnv, MarketMakingEnv, MultiAgentEnv
    mm = lambda env, g: env.step(torch.randint(0, 5, (4, 1, 2), generator=g))
    kw = dict(n_envs=4, msgs_per_step=5, seed=1, action_space="spread_skew", reward_function="spooner",
              unwind_price="far_touch")
    cpu, rc = _run(MarketMakingEnv, "cpu", mm, **kw)
    gpu, rg = _run(MarketMakingEnv, "cuda", mm, **kw)
    assert gpu.engine.on_gpu and torch.equal(rc, rg)
    assert torch.equal(cpu.inv, gpu.inv) and torch.equal(cpu.cash, gpu.cash)
    ex = lambda env, g: env.step(torch.randint(0, 13, (4,), generator=g))
    kw = dict(n_envs=4, msgs_per_step=5, seed=1, target=300, task="random", action_space="fixed_quants_complex",
              reward_function="normal")
    cpu, rc = _run(ExecutionEnv, "cpu", ex, **kw)
    gpu, rg = _run(ExecutionEnv, "cuda", ex, **kw)
    assert torch.equal(rc, rg) and torch.equal(cpu.done_qty, gpu.done_qty)
    ma = lambda env, g: env.step(torch.randint(0, 5, (4, 2, 2), generator=g),
                                 exec_actions=torch.randint(0, 6, (4, 1), generator=g))
    kw = dict(n_envs=4, msgs_per_step=5, seed=1, n_mm=2, n_exec=1, exec_action_space="fixed_quants",
              action_space="offsets", shuffle_action_messages=True)
    cpu, rc = _run(MultiAgentEnv, "cpu", ma, **kw)
    gpu, rg = _run(MultiAgentEnv, "cuda", ma, **kw)
    assert torch.equal(rc, rg) and torch.equal(cpu.exec_done, gpu.exec_done)
