"""State model: frames, chart coordinates, FrameDiT, rectified flow, pretraining."""
import numpy as np
import pytest
import torch

from sigma0_b200.data.synthetic import generate_day
from sigma0_b200.state import (BookDiT, ChartNormalizer, FrameDiT, FrameDiTConfig, FrameWindowDataset,
                               RectifiedFlow, bind_condition, bind_unconditional, decode_frames,
                               decode_frames_torch, encode_frames, encode_series, eps_from_v, fit_normalizer,
                               flow_matching_loss, interpolate, load_checkpoint, pretrain_step,
                               resample_events, resample_wide_book, sample, sample_context_masks,
                               save_checkpoint, score_from_v, velocity_target, x0_from_v)


def test_resample_forward_fills_and_counts():
    t = np.array([5, 7, 7, 23, 31], dtype=np.int64)
    st = np.arange(5, dtype=np.float32)[:, None] * np.ones((1, 4), np.float32)
    fs = resample_events(t, st, interval_ns=10)
    assert fs.times_ns.tolist() == [10, 20, 30]
    assert fs.frames[:, 0].tolist() == [2, 2, 3]          # last event at or before 10, 20, 30
    assert fs.events_per_frame.tolist() == [3, 0, 1]
    assert fs.horizon_ns == 30
    with pytest.raises(ValueError):
        resample_events(t[::-1].copy(), st, 10)


def test_chart_round_trip_and_noise_decodes_valid():
    d = generate_day(400, seed=3)
    fs = resample_wide_book(d.books, interval_ns=2_000_000)
    chart, anchor = encode_frames(fs.frames, fs.events_per_frame)
    assert chart.shape[1] == fs.frames.shape[1] + 1
    back = decode_frames(chart, anchor)
    assert np.allclose(back, fs.frames, atol=1e-2 * np.abs(fs.frames).max())
    noise = np.random.default_rng(0).normal(size=(50, chart.shape[1])).astype(np.float32)
    book = decode_frames(noise, 1000.0)
    assert (book[:, 0] > book[:, 2]).all()
    assert (np.diff(book[:, 0::4], axis=1) > 0).all() and (np.diff(book[:, 2::4], axis=1) < 0).all()
    ct = torch.from_numpy(chart[None]).double().requires_grad_(True)
    bt = decode_frames_torch(ct, torch.tensor([anchor], dtype=torch.float64))
    assert np.allclose(bt[0].detach().numpy(), back, atol=1e-3 * np.abs(back).max())
    bt.sum().backward()
    assert torch.isfinite(ct.grad).all()


def test_normalizer_round_trip():
    c = np.random.default_rng(1).normal(3, 2, size=(100, 9)).astype(np.float32)
    n = ChartNormalizer.fit(c)
    assert np.allclose(n.denormalize(n.normalize(c)), c, atol=1e-5)
    n2 = ChartNormalizer.from_state_dict(n.state_dict())
    assert np.allclose(n2.mean, n.mean)


def test_conversion_identities_and_sde_degenerates_to_ode():
    torch.manual_seed(0)
    x0, eps = torch.randn(3, 5, 4), torch.randn(3, 5, 4)
    t = torch.rand(3) * 0.9 + 0.05
    x_t = interpolate(x0, eps, t)
    v = velocity_target(x0, eps)
    assert torch.allclose(x0_from_v(x_t, v, t), x0, atol=1e-5)
    assert torch.allclose(eps_from_v(x_t, v, t), eps, atol=1e-5)
    assert torch.allclose(score_from_v(x_t, v, t), -eps / t.view(-1, 1, 1), atol=1e-4)
    fn = lambda x, tt: 0.3 * x
    g1, g2 = torch.Generator().manual_seed(1), torch.Generator().manual_seed(1)
    a = RectifiedFlow(8).sample_ode(fn, (2, 5, 4), "cpu", generator=g1)
    b, recs = RectifiedFlow(8, noise_scale=0.0).sample_sde_trajectory(fn, (2, 5, 4), "cpu", generator=g2)
    assert torch.allclose(a, b) and len(recs) == 8
    with pytest.raises(ValueError):
        RectifiedFlow(8).step_log_prob(fn, recs[0])


def test_framedit_parameter_account_and_zero_init():
    m = FrameDiT(FrameDiTConfig(channels=41, hidden=128, depth=4, heads=4, conditional=False))
    assert sum(p.numel() for p in m.parameters()) == 953_769
    mc = FrameDiT(FrameDiTConfig(channels=8, hidden=32, depth=1, heads=2, max_seq_len=16))
    assert (mc.input_proj.weight[:, 8:] == 0).all()
    x = torch.randn(2, 6, 8)
    fn = bind_condition(mc, torch.randn(2, 6, 8), torch.ones(2, 6))
    assert (fn(x, torch.rand(2)) == 0).all()                        # zero-init velocity head
    assert bind_unconditional(mc)(x, torch.rand(2)).shape == x.shape
    with pytest.raises(ValueError):
        FrameDiT(FrameDiTConfig(channels=8, hidden=32, depth=1, heads=2, max_seq_len=4))(
            torch.randn(1, 6, 17), torch.rand(1))


def test_context_masks_are_per_sample_prefixes():
    m = sample_context_masks(64, 10, 6, generator=torch.Generator().manual_seed(0))
    assert m.shape == (64, 10)
    assert (m[:, 1:] <= m[:, :-1]).all()                           # prefixes
    assert len(set(m.sum(1).tolist())) > 1 and m.sum(1).max() <= 6


def test_pretraining_learns_and_checkpoints(tmp_path):
    torch.manual_seed(0)
    d = generate_day(3000, seed=5)
    fs = resample_wide_book(d.books, interval_ns=1_000_000)
    norm = fit_normalizer([fs])
    ds = FrameWindowDataset([encode_series(fs, norm)], seq_len=16, stride=8)
    x0 = torch.stack([ds[i][0] for i in range(min(len(ds), 32))])
    cfg = FrameDiTConfig(channels=x0.shape[-1], hidden=32, depth=2, heads=2, max_seq_len=16)
    model = FrameDiT(cfg)
    opt = torch.optim.Adam(model.parameters(), lr=3e-3)
    losses = []
    for _ in range(60):
        out = pretrain_step(model, x0, max_ctx=8)
        opt.zero_grad(); out["loss"].backward(); opt.step()
        losses.append(float(out["loss"]))
    assert np.mean(losses[-10:]) < np.mean(losses[:10])
    save_checkpoint(str(tmp_path), 60, model, opt, norm, cfg)
    m2 = FrameDiT(cfg)
    assert load_checkpoint(str(tmp_path), m2) == 60
    for a, b in zip(model.state_dict().values(), m2.state_dict().values()):
        assert torch.equal(a, b)


def test_bookdit_flow_matching_learns_and_samples():
    torch.manual_seed(0)
    C, T, K = 8, 16, 4
    model = BookDiT(C, T, K, d=64, depth=2, heads=4)
    opt = torch.optim.Adam(model.parameters(), lr=2e-3)
    ctx = torch.randn(64, K, C)
    x0 = ctx.mean(1, keepdim=True).expand(-1, T, -1) + 0.05 * torch.randn(64, T, C)
    losses = []
    for _ in range(60):
        loss = flow_matching_loss(model, x0, ctx)
        opt.zero_grad(); loss.backward(); opt.step()
        losses.append(float(loss))
    assert np.mean(losses[-10:]) < np.mean(losses[:10])
    s = sample(model, ctx[:4], steps=8)
    assert s.shape == (4, T, C) and torch.isfinite(s).all()
