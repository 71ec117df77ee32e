"""The S5 complex diagonal scan kernels (csrc/s5_scan.cu) against the chunked einsum path
of the same module: outputs and the gradients of every parameter and the input, for the
causal and bidirectional layers, ragged lengths and a carried initial state."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a - b).abs().norm() / b.abs().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("L,bidir", [(300, False), (1000, True), (64, False)])
def test_s5_scan_matches_einsum_path(L, bidir):
    from sigma0_b200.models.s5 import make_s5_factory
    torch.manual_seed(L)
    m = make_s5_factory(64, 2, bidirectional=bidir)(48).cuda()
    u = torch.randn(3, L, 48, device="cuda", requires_grad=True)
    y1 = m(u)
    g = torch.randn_like(y1)
    grads1 = torch.autograd.grad((y1 * g).sum(), [u] + list(m.parameters()))
    m.use_kernel = False
    y2 = m(u)
    grads2 = torch.autograd.grad((y2 * g).sum(), [u] + list(m.parameters()))
    assert _rel(y1, y2) < 1e-4
    for (name, _), a, b in zip([("u", None)] + list(m.named_parameters()), grads1, grads2):
        assert _rel(a, b) < 1e-3, (name, _rel(a, b))


def test_s5_step_with_state_matches():
    from sigma0_b200.models.s5 import make_s5_factory
    torch.manual_seed(0)
    m = make_s5_factory(64, 2)(48).cuda()
    u = torch.randn(2, 130, 48, device="cuda")
    x0 = m.initial_state(2, "cuda") + 0.3 * torch.randn(2, m.P, dtype=torch.complex64, device="cuda")
    x1, y1 = m.step(x0, u)
    m.use_kernel = False
    x2, y2 = m.step(x0, u)
    assert _rel(y1, y2) < 1e-4 and _rel(x1, x2) < 1e-4
