"""Randomized shapes (hypothesis) for the attention, S5 and gated-delta kernels against
their oracles, and determinism of the forward kernels that use no atomics (two runs,
bit-identical outputs)."""
import pytest
import torch
from hypothesis import HealthCheck, given, settings, strategies as st

pytestmark = pytest.mark.gpu

SETTINGS = dict(max_examples=8, deadline=None, suppress_health_check=list(HealthCheck), derandomize=True)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@settings(**SETTINGS)
@given(B=st.integers(1, 2), Lq=st.integers(1, 300), extra=st.integers(0, 200), nh=st.integers(1, 3),
       hd=st.sampled_from([64, 128]), window=st.one_of(st.none(), st.integers(1, 150)))
def test_attention_random_shapes(B, Lq, extra, nh, hd, window):
    from sigma0_b200.ops.attention import flash_attention
    Lk = Lq + extra
    g = torch.Generator(device="cuda").manual_seed(Lq * 31 + extra)
    q = torch.randn(B, Lq, nh, hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Lk, nh, hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Lk, nh, hd, device="cuda", generator=g).to(torch.bfloat16)
    o = flash_attention(q, k, v, window=window, q_offset=extra, force_kernel=True)
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    s = qf @ kf.transpose(-1, -2) * hd ** -0.5
    qpos = extra + torch.arange(Lq, device="cuda")[:, None]
    kpos = torch.arange(Lk, device="cuda")[None]
    m = kpos <= qpos
    if window:
        m &= kpos > qpos - window
    ref = (torch.softmax(s.masked_fill(~m, float("-inf")), -1).nan_to_num(0.0) @ vf).transpose(1, 2)
    assert _rel(o, ref) < 1e-2


@settings(**SETTINGS)
@given(L=st.integers(1, 400), blocks=st.sampled_from([1, 2, 4]), bidir=st.booleans())
def test_s5_random_lengths(L, blocks, bidir):
    from sigma0_b200.models.s5 import make_s5_factory
    torch.manual_seed(L)
    m = make_s5_factory(32, blocks, bidirectional=bidir)(24).cuda()
    u = torch.randn(2, L, 24, device="cuda")
    y1 = m(u)
    m.use_kernel = False
    y2 = m(u)
    assert _rel(y1, y2) < 1e-4


@settings(**SETTINGS)
@given(L=st.integers(1, 300), kda=st.booleans(), hd=st.sampled_from([64, 128]))
def test_gated_delta_random_lengths(L, kda, hd):
    from sigma0_b200.models.gdn import gated_delta_chunked, l2_normalize
    g = torch.Generator(device="cuda").manual_seed(L + hd)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    q, k = l2_normalize(r(1, L, 2, hd)) * hd ** -0.5, l2_normalize(r(1, L, 2, hd))
    v, beta = r(1, L, 2, 64), torch.sigmoid(r(1, L, 2))
    alog = torch.nn.functional.logsigmoid(r(1, L, 2, hd if kda else 1) + 3.0)
    o1, S1 = gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=True)
    o2, S2 = gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=False)
    assert _rel(o1, o2) < 2e-2 and _rel(S1, S2) < 2e-2


def test_forward_kernels_are_deterministic():
    """Kernels without atomics give bit-identical results on a second run."""
    from sigma0_b200.models.gdn import gated_delta_chunked, l2_normalize
    from sigma0_b200.models.s5 import make_s5_factory
    from sigma0_b200.ops.attention import flash_attention
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(2, 700, 4, 64, device="cuda", generator=g).to(torch.bfloat16)
    a1 = flash_attention(q, q, q, window=200)
    a2 = flash_attention(q, q, q, window=200)
    assert torch.equal(a1, a2)
    m = make_s5_factory(64, 2)(48).cuda()
    u = torch.randn(2, 500, 48, device="cuda", generator=g)
    assert torch.equal(m(u), m(u))
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    args = (l2_normalize(r(1, 500, 2, 128)), l2_normalize(r(1, 500, 2, 128)), r(1, 500, 2, 256),
            torch.sigmoid(r(1, 500, 2)), torch.nn.functional.logsigmoid(r(1, 500, 2, 1) + 3))
    o1, S1 = gated_delta_chunked(*args, 64, use_kernel=True)
    o2, S2 = gated_delta_chunked(*args, 64, use_kernel=True)
    assert torch.equal(o1, o2) and torch.equal(S1, S2)
