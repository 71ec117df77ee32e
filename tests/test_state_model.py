"""Book-state world model: frames, chart round trip, flow-matching training and sampling."""
import numpy as np
import torch

from sigma0_b200.data.synthetic import generate_day
from sigma0_b200.state import (BookDiT, decode_chart, encode_chart, flow_matching_loss, resample_frames,
                               reward_weighted_loss, sample, smoothness_reward)


def test_frames_and_chart_round_trip():
    d = generate_day(300, seed=3)
    frames, counts = resample_frames(d.books, interval_ns=2_000_000)
    assert counts.sum() <= len(d.books) and frames.shape[1] == 40
    chart, anchor = encode_chart(frames)
    back = decode_chart(chart, anchor)
    assert np.allclose(back[:, 1::4], frames[:, 1::4]) and np.allclose(back[:, 3::4], frames[:, 3::4])
    assert np.allclose(back[:, 0] - back[:, 2], frames[:, 0] - frames[:, 2])


def test_flow_matching_learns_and_samples():
    torch.manual_seed(0)
    C, T, K = 8, 16, 4
    model = BookDiT(C, T, K, d=64, depth=2, heads=4)
    opt = torch.optim.Adam(model.parameters(), lr=2e-3)
    # data: a constant per-sample offset plus small noise, conditioned on the context mean
    ctx = torch.randn(64, K, C)
    x1 = ctx.mean(1, keepdim=True).expand(-1, T, -1) + 0.05 * torch.randn(64, T, C)
    losses = []
    for _ in range(60):
        loss = flow_matching_loss(model, x1, ctx)
        opt.zero_grad(); loss.backward(); opt.step()
        losses.append(float(loss))
    assert np.mean(losses[-10:]) < np.mean(losses[:10])
    s = sample(model, ctx[:4], steps=8)
    assert s.shape == (4, T, C) and torch.isfinite(s).all()
    lw, r = reward_weighted_loss(model, ctx[:4], smoothness_reward, n_samples=3, steps=4)
    assert torch.isfinite(lw) and torch.isfinite(r)
