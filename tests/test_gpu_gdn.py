"""The gated-delta-rule chunk scan kernels (csrc/gdn_scan.cu) against the host-loop
oracle of ``gated_delta_chunked``: outputs, final state and the gradients of q, k, v,
beta, the decay logits and the initial state, for GDN (per-head decay) and KDA
(per-key-dim decay), head dims 64 and 128, ragged lengths."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, L, nh, hd, hvd, kda, seed):
    from sigma0_b200.models.gdn import l2_normalize
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    q = l2_normalize(r(B, L, nh, hd)) * hd ** -0.5
    k = l2_normalize(r(B, L, nh, hd))
    v = r(B, L, nh, hvd)
    beta = torch.sigmoid(r(B, L, nh))
    alog = torch.nn.functional.logsigmoid(r(B, L, nh, hd if kda else 1) + 3.0)
    S0 = 0.1 * r(B, nh, hvd, hd)
    return [t.requires_grad_(True) for t in (q, k, v, beta, alog, S0)]


def _rel(a, b):
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("B,L,nh,hd,hvd,kda", [(2, 200, 2, 64, 128, False), (1, 300, 2, 128, 256, True),
                                               (1, 64, 1, 128, 64, False)])
def test_gdn_scan_matches_host_loop(B, L, nh, hd, hvd, kda):
    from sigma0_b200.models.gdn import gated_delta_chunked
    xs = _inputs(B, L, nh, hd, hvd, kda, L + hd)
    ys = [x.detach().clone().requires_grad_(True) for x in xs]
    o1, S1 = gated_delta_chunked(*xs[:5], S0=xs[5], use_kernel=True)
    o2, S2 = gated_delta_chunked(*ys[:5], S0=ys[5], use_kernel=False)
    assert _rel(o1, o2) < 2e-2 and _rel(S1, S2) < 2e-2, (_rel(o1, o2), _rel(S1, S2))
    g = torch.Generator(device="cuda").manual_seed(1)
    wo, ws = torch.randn(o2.shape, device="cuda", generator=g), torch.randn(S2.shape, device="cuda", generator=g)
    ((o1 * wo).sum() + (S1 * ws).sum()).backward()
    ((o2 * wo).sum() + (S2 * ws).sum()).backward()
    for name, a, b in zip(("q", "k", "v", "beta", "alog", "S0"), xs, ys):
        assert _rel(a.grad, b.grad) < 3e-2, (name, _rel(a.grad, b.grad))


def test_gdn_layer_uses_the_scan_kernel():
    from sigma0_b200.models.gdn import GDN
    from sigma0_b200.ops import _ext
    m = GDN(256, num_heads=2, head_dim=64).cuda()
    _ext.reset_launch_count()
    m(torch.randn(1, 130, 256, device="cuda")).sum().backward()
    assert _ext.launch_count() >= 2


def test_kda_intra_kernel_matches_einsum():
    """Per-key-dim decay score / WY matrices and their gradients against the tensor
    expression (strong decays included: the weights stay in [0, 1])."""
    from sigma0_b200.models.gdn import _KDAIntra
    g = torch.Generator(device="cuda").manual_seed(3)
    N, C, hd = 6, 64, 128
    q, k, kb = (torch.randn(N, C, hd, device="cuda", generator=g).requires_grad_(True) for _ in range(3))
    alog = torch.nn.functional.logsigmoid(torch.randn(N, C, hd, device="cuda", generator=g) * 3)
    G = alog.cumsum(1).requires_grad_(True)
    I1, L1 = _KDAIntra.apply(q, k, kb, G)
    xs = [t.detach().clone().requires_grad_(True) for t in (q, k, kb, G)]
    tri = torch.tril(torch.ones(C, C, dtype=torch.bool, device="cuda"))
    W = torch.exp((xs[3][:, :, None, :] - xs[3][:, None, :, :]).masked_fill(~tri[..., None], 0.0)) * tri[..., None]
    I2 = torch.einsum("nid,njd,nijd->nij", xs[0], xs[1], W)
    L2 = -torch.einsum("nid,njd,nijd->nij", xs[2], xs[1], W) * torch.tril(tri, -1)
    assert _rel(I1, I2) < 1e-4 and _rel(L1, L2) < 1e-4
    wI, wL = torch.randn_like(I2), torch.randn_like(L2)
    ((I1 * wI).sum() + (L1 * wL).sum()).backward()
    ((I2 * wI).sum() + (L2 * wL).sum()).backward()
    for name, a, b in zip(("q", "k", "kb", "G"), (q, k, kb, G), xs):
        assert _rel(a.grad, b.grad) < 1e-4, (name, _rel(a.grad, b.grad))


def test_segment_transition_with_the_scan_kernels():
    """The final state from an initial state S0 equals S0 T + the final state from zero
    (the identity context parallelism composes segments with), with the CUDA scans."""
    from sigma0_b200.models.gdn import gated_delta_chunked
    for kda in (False, True):
        q, k, v, beta, alog, S0 = (t.detach() for t in _inputs(1, 200, 2, 128, 128, kda, 7))
        _, S_zero, T = gated_delta_chunked(q, k, v, beta, alog, 64, use_kernel=True, return_transition=True)
        _, S_full = gated_delta_chunked(q, k, v, beta, alog, 64, S0=S0, use_kernel=True)
        assert _rel(S_full, S0 @ T + S_zero) < 2e-2


@pytest.mark.parametrize("kda,hd,T", [(False, 128, 1), (True, 64, 5), (False, 64, 3)])
def test_decode_kernel_matches_recurrence(kda, hd, T):
    """The gdn_decode kernel against the token loop: outputs and the updated state, from a
    non-zero state, over several tokens per call."""
    from sigma0_b200.models.gdn import gated_delta_recurrent
    q, k, v, beta, alog, S0 = (t.detach() for t in _inputs(3, T, 4, hd, 2 * hd, kda, T + hd))
    o1, S1 = gated_delta_recurrent(q, k, v, beta, alog, S0, use_kernel=True)
    o2, S2 = gated_delta_recurrent(q, k, v, beta, alog, S0, use_kernel=False)
    assert _rel(o1, o2) < 1e-4 and _rel(S1, S2) < 1e-4
    assert not torch.equal(S0, S1)                 # the input state is left untouched, a new one returned


@pytest.mark.parametrize("kda", [False, True])
def test_gdn_module_step_matches_forward(kda):
    """Stepping a GDN / KDA mixer token by token on CUDA (decode kernel, convolution buffers)
    reproduces its full-sequence forward."""
    from sigma0_b200.models.gdn import GDN
    torch.manual_seed(0)
    m = GDN(256, num_heads=4, head_dim=64, use_kda=kda).cuda()
    x = torch.randn(2, 70, 256, device="cuda")
    with torch.no_grad():
        full = m(x)
        st = m.initial_state(2, "cuda")
        outs = []
        for t in range(70):
            st, y = m.step(st, x[:, t:t + 1])
            outs.append(y)
    assert _rel(torch.cat(outs, 1), full) < 2e-2
