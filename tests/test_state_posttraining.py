"""Post-training trainers and rewards of the state model: one step each plus contracts."""
import pytest
import torch

from sigma0_b200.state import (AWMTrainer, BookValidityReward, DMDRTrainer, DMDTrainer, FlowGRPOTrainer, FrameDiT,
                               FrameDiTConfig, RAMTrainer, RectifiedFlow, ReFLTrainer, ReturnSanityReward,
                               bind_unconditional, default_rule_reward, make_repaint_pin)

LEVELS = 2
C = 4 * LEVELS
SHAPE = (6, C)


def tiny(seed=0):
    torch.manual_seed(seed)
    m = FrameDiT(FrameDiTConfig(channels=C, hidden=32, depth=1, heads=2, max_seq_len=16, conditional=False))
    with torch.no_grad():
        m.velocity_head.weight.add_(0.01 * torch.randn_like(m.velocity_head.weight))
    return m


def has_grad(m):
    return any(p.grad is not None and p.grad.abs().sum() > 0 for p in m.parameters())


def soft_reward(frames):
    return torch.sigmoid(frames[..., 0]).flatten(1).mean(1)


def book(crossed=False):
    b = torch.zeros(1, 4, C)
    a0, b0 = (99.0, 101.0) if crossed else (101.0, 99.0)
    for k in range(LEVELS):
        b[..., 4 * k], b[..., 4 * k + 1] = a0 + 2 * k, 10.0
        b[..., 4 * k + 2], b[..., 4 * k + 3] = b0 - 2 * k, 10.0
    return b


def test_rewards():
    r = BookValidityReward()
    assert r(book()).item() == pytest.approx(1.0) and r(book(True)).item() < 1.0
    x = book(True).requires_grad_(True)
    BookValidityReward(soft=True)(x).sum().backward()
    assert torch.isfinite(x.grad).all() and x.grad.abs().sum() > 0
    wild = book().clone()
    wild[:, 2:, 0] += 500.0
    wild[:, 2:, 2] += 500.0
    assert ReturnSanityReward()(wild).item() < ReturnSanityReward()(book()).item()
    assert 0.0 < default_rule_reward()(book()).item() <= 1.0


def test_refl_backpropagates_reward():
    m = tiny()
    out = ReFLTrainer(m, RectifiedFlow(6), soft_reward, fm_weight=0.1).step(
        (4, *SHAPE), "cpu", data_batch=torch.randn(4, *SHAPE))
    out["loss"].backward()
    assert torch.isfinite(out["loss"]) and has_grad(m)


def test_grpo_needs_noise_learns_and_flat_reward_is_neutral():
    m = tiny()
    with pytest.raises(ValueError):
        FlowGRPOTrainer(m, RectifiedFlow(6), soft_reward)
    flow = RectifiedFlow(6, noise_scale=0.3)
    out = FlowGRPOTrainer(m, flow, soft_reward, group_size=4, timestep_fraction=0.5).step(SHAPE, "cpu")
    out["loss"].backward()
    assert has_grad(m) and out["ratio_mean"].item() == pytest.approx(1.0)
    flat = FlowGRPOTrainer(m, flow, lambda f: torch.ones(f.shape[0]), group_size=4).step(SHAPE, "cpu")
    assert abs(flat["loss"].item()) < 1e-6
    with pytest.raises(ValueError):       # a pin without a frame mask
        FlowGRPOTrainer(m, flow, soft_reward, group_size=4).step(
            SHAPE, "cpu", pin=make_repaint_pin(torch.zeros(4, *SHAPE), torch.ones(4, SHAPE[0])))


def test_awm_learns_anchor_and_flat_reward():
    m = tiny()
    tr = AWMTrainer(m, RectifiedFlow(6), soft_reward, group_size=4, n_noise_draws=2)
    out = tr.step(SHAPE, "cpu")
    out["loss"].backward()
    assert has_grad(m)
    tr2 = AWMTrainer(m, RectifiedFlow(6), soft_reward, group_size=4, n_noise_draws=1, fm_anchor_weight=0.5)
    out2 = tr2.step(SHAPE, "cpu", data_batch=torch.randn(3, *SHAPE))
    assert out2["fm_anchor"].item() > 0
    flat = AWMTrainer(m, RectifiedFlow(6), lambda f: torch.ones(f.shape[0]), group_size=4).step(SHAPE, "cpu")
    assert abs(flat["loss"].item()) < 1e-6


def test_ram_moves_only_bad_endpoints_and_learns():
    m = tiny()
    tr = RAMTrainer(m, RectifiedFlow(6), soft_reward, group_size=4, beta=1.0, temperature=0.01)
    x0 = torch.randn(4, *SHAPE)
    r = torch.tensor([0.0, 0.2, 0.5, 1.0])
    adj, rt = tr.adjusted_endpoints(x0, r)
    assert torch.allclose(adj[3], x0[3], atol=1e-4)                 # the best one keeps its endpoint
    assert torch.allclose(adj[0], x0[3], atol=1e-3)                 # the worst moves to the (sharp) centroid
    out = tr.step(SHAPE, "cpu")
    out["loss"].backward()
    assert has_grad(m)


def test_dmd_moves_student_not_teacher_and_dmdr_adds_reward():
    student, teacher, fake = tiny(0), tiny(1), tiny(2)
    for p in teacher.parameters():
        p.requires_grad_(False)
    tr = DMDTrainer(student, teacher, fake, RectifiedFlow(4), student_steps=2)
    out = tr.step(SHAPE, "cpu", batch_size=3)
    (out["loss_student"] + out["loss_fake"]).backward()
    assert has_grad(student) and has_grad(fake) and not has_grad(teacher)
    with pytest.raises(ValueError):
        DMDTrainer(student, teacher, fake, RectifiedFlow(4), n_blocks=2)
    two = DMDTrainer(student, teacher, fake, RectifiedFlow(4), student_steps=2, n_blocks=2,
                     rebind=lambda prev: bind_unconditional(student))
    assert two.rollout((2, *SHAPE), "cpu").shape == (2, 2 * SHAPE[0], C)
    r = DMDRTrainer(student, teacher, fake, RectifiedFlow(4), student_steps=2, reward=soft_reward)
    o = r.step(SHAPE, "cpu", batch_size=2)
    assert "reward_mean" in o and torch.isfinite(o["loss_student"])
