"""The sm_100a flash attention kernels (csrc/attention.cu) against an fp32 torch
restatement: causal, sliding window, decode offsets, strided q/k/v views, head dims 64
and 128, forward and all three gradients."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale, window, q_offset):
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    s = qf @ kf.transpose(-1, -2) * scale
    Lq, Lk = q.shape[1], k.shape[1]
    qpos = q_offset + torch.arange(Lq, device=q.device)[:, None]
    kpos = torch.arange(Lk, device=q.device)[None, :]
    m = kpos <= qpos
    if window:
        m &= kpos > qpos - window
    p = torch.softmax(s.masked_fill(~m, float("-inf")), -1).nan_to_num(0.0)
    return (p @ vf).transpose(1, 2)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


CASES = [  # B, Lq, Lk, nh, hd, window, q_offset
    (2, 300, 300, 3, 64, None, 0),
    (1, 517, 517, 2, 128, None, 0),
    (2, 400, 400, 2, 64, 100, 0),
    (1, 333, 333, 2, 128, 64, 0),
    (2, 7, 250, 2, 64, None, 243),
    (1, 26, 700, 2, 128, 130, 674),
    (1, 128, 128, 1, 64, None, 0),
]


@pytest.mark.parametrize("B,Lq,Lk,nh,hd,window,q_offset", CASES)
def test_flash_attention_forward_backward(B, Lq, Lk, nh, hd, window, q_offset):
    from sigma0_b200.ops.attention import flash_attention
    torch.manual_seed(Lq * 7 + hd + (window or 0))
    dev = "cuda"
    # q from a fused [B, L, 3, nh, hd] projection: strided views, as the models produce
    qkv = torch.randn(B, Lk, 3, nh, hd, device=dev).to(torch.bfloat16)
    q = qkv[:, Lk - Lq:, 0].detach().requires_grad_(True)
    k = qkv[:, :, 1].detach().requires_grad_(True)
    v = qkv[:, :, 2].detach().requires_grad_(True)
    scale = hd ** -0.5
    o = flash_attention(q, k, v, scale=scale, window=window, q_offset=q_offset, force_kernel=True)
    qr, kr, vr = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    ref = _ref(qr, kr, vr, scale, window, q_offset)
    assert _rel(o, ref) < 1e-2
    do = torch.randn_like(ref)
    (o.float() * do).sum().backward()
    (ref * do).sum().backward()
    for name, a, b in (("dq", q.grad, qr.grad), ("dk", k.grad, kr.grad), ("dv", v.grad, vr.grad)):
        assert _rel(a, b) < 2e-2, (name, _rel(a, b))


def test_flash_attention_runs_the_kernel():
    from sigma0_b200.ops import _ext
    from sigma0_b200.ops.attention import flash_attention
    q = torch.randn(1, 64, 2, 64, device="cuda", dtype=torch.bfloat16)
    before = _ext.launch_count() if hasattr(_ext, "launch_count") else None
    flash_attention(q, q, q, window=32)
    torch.cuda.synchronize()
    if before is not None:
        assert _ext.launch_count() > before

