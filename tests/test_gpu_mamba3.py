"""GPU numerics of the Mamba3 kernels against the plain-torch fp32 oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _layer(H=512, seed=0):
    from sigma0_b200.models.mamba3 import Mamba3
    torch.manual_seed(seed)
    m = Mamba3(H, impl="cuda").cuda()
    with torch.no_grad():
        m.B_bias.normal_(0, 0.5)
        m.C_bias.normal_(0, 0.5)
        m.D.normal_(1, 0.2)
        m.B_norm.scale.normal_(1, 0.1)
        m.C_norm.scale.normal_(1, 0.1)
        m.in_proj.kernel.mul_(2.0)
    return m


def _oracle_y(m, proj, B, L):
    from sigma0_b200.ops.reference import mamba3_ref as ref
    z, x, Bn, Cn, ADT, DT, trap, ang = m._prep(proj.float().view(B, L, -1))
    nh = m.dims.n_heads
    Bh = Bn[:, :, None, :].expand(-1, -1, nh, -1)
    Ch = Cn[:, :, None, :].expand(-1, -1, nh, -1)
    y = ref.mamba3_ssd_chunked(Ch, Bh, x, ADT.transpose(1, 2), DT.transpose(1, 2), trap.transpose(1, 2),
                               ang, m.C_bias, m.B_bias, m.D, z, chunk_size=64)
    return y.reshape(B, L, -1)


@pytest.mark.parametrize("L", [64, 200, 1000])
def test_ssd_forward_matches_oracle(L):
    from sigma0_b200.ops._ext import ext
    C = ext()
    m = _layer()
    B = 2
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    proj = (torch.randn(B * L, ldp, device="cuda") * 0.5).to(torch.bfloat16)
    y = C.m3_fwd(proj, B, L, d.n_heads, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D,
                 m.A_floor, 1e-6)[0]
    yr = _oracle_y(m, proj[:, :d.d_in_proj].contiguous(), B, L)
    assert torch.isfinite(y.float()).all()
    assert rel(y, yr) < 2e-2, rel(y, yr)


def _walker_args(B, L, H, seed):
    m = _layer(H=H, seed=seed)
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    proj = (torch.randn(B * L, ldp, device="cuda") * 0.5).to(torch.bfloat16)
    proj[:, d.d_in_proj:] = 0
    return m, d, proj


@pytest.mark.parametrize("B,L,H", [(2, 64, 512), (3, 200, 512), (1, 1000, 256), (2, 4100, 512)])
def test_ssd_forward_walker_matches_chunk_parallel_kernels(B, L, H):
    """The tcgen05 chunk walker against the chunk-parallel kernels: y, final state and angle."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    m, d, proj = _walker_args(B, L, H, 2)
    args = (proj, B, L, d.n_heads, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D,
            m.A_floor, 1e-6, True)
    st = C.m3_tc_status(proj)
    st.zero_()
    try:
        C.m3_use_tc(False)
        y0, _, f0, th0 = C.m3_fwd(*args)[:4]
        C.m3_use_tc(True)
        y1, _, f1, th1 = C.m3_fwd(*args)[:4]
    finally:
        C.m3_use_tc(None)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.isfinite(y1.float()).all()
    assert rel(y1, y0) < 1e-2, rel(y1, y0)
    assert rel(f1, f0) < 1e-2, rel(f1, f0)
    dth = torch.remainder(th1 - th0 + 3.14159265, 2 * 3.14159265) - 3.14159265
    assert dth.abs().max().item() < 1e-3


@pytest.mark.parametrize("B,L,H", [(2, 64, 512), (3, 200, 512), (1, 1000, 256), (2, 2100, 512)])
def test_ssd_backward_walker_matches_chunk_parallel_kernels(B, L, H):
    """The reverse tcgen05 walker (given the forward walker's saved images) against the
    chunk-parallel backward kernels: every output of m3_bwd."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    m, d, proj = _walker_args(B, L, H, 3)
    dy = torch.randn(B, L, d.d_inner, device="cuda").to(torch.bfloat16)
    common = (m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D)
    st = C.m3_tc_status(proj)
    st.zero_()
    try:
        C.m3_use_tc(False)
        ref = C.m3_bwd(proj, dy, *common, B, L, d.n_heads, m.A_floor, 1e-6)
        C.m3_use_tc(True)
        out = C.m3_fwd(proj, B, L, d.n_heads, *common, m.A_floor, 1e-6, False, True)
        got = C.m3_bwd(proj, dy, *common, B, L, d.n_heads, m.A_floor, 1e-6, saved_states=out[1],
                       saved_prep=list(out[4:]))
    finally:
        C.m3_use_tc(None)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    names = ["dproj", "dwB", "dwC", "ddt_bias", "dD", "dC_bias", "dB_bias"]
    for name, a, b in zip(names, got, ref):
        assert torch.isfinite(a.float()).all(), name
        assert rel(a, b) < 2e-2, (name, rel(a, b))


@pytest.mark.parametrize("B,L,nseg", [(1, 1000, 3), (2, 4100, 5), (1, 300, 5)])
def test_ssd_walkers_split_into_segments_match_one_walk(B, L, nseg, monkeypatch):
    """Sequences cut into segments (walked in parallel, then re-walked from the carried state /
    gradient) give the single walk's forward and backward outputs."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    m, d, proj = _walker_args(B, L, 512, 5)
    dy = torch.randn(B, L, d.d_inner, device="cuda").to(torch.bfloat16)
    common = (m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D)
    res = {}
    C.m3_use_tc(True)
    try:
        for k in (1, nseg):
            monkeypatch.setenv("S0_M3_SEGMENTS", str(k))
            out = C.m3_fwd(proj, B, L, d.n_heads, *common, m.A_floor, 1e-6, True, True)
            y, st, fin, thf = out[:4]
            res[k] = (y, fin, thf) + tuple(C.m3_bwd(proj, dy, *common, B, L, d.n_heads, m.A_floor, 1e-6,
                                                     saved_states=st, saved_prep=list(out[4:])))
    finally:
        C.m3_use_tc(None)
    torch.cuda.synchronize()
    assert int(C.m3_tc_status(proj).item()) == 0
    names = ["y", "fin", "thf", "dproj", "dwB", "dwC", "ddt_bias", "dD", "dC_bias", "dB_bias"]
    for name, a, b in zip(names, res[nseg], res[1]):
        if name == "thf":
            dth = torch.remainder(a - b + 3.14159265, 2 * 3.14159265) - 3.14159265
            assert dth.abs().max().item() < 1e-3
            continue
        assert rel(a, b) < 1e-2, (name, rel(a, b))


@pytest.mark.parametrize("L", [128, 150, 700])
def test_ssd_backward_matches_oracle(L):
    from sigma0_b200.ops._ext import ext
    C = ext()
    m = _layer(seed=1)
    B = 2
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    proj = (torch.randn(B * L, ldp, device="cuda") * 0.5).to(torch.bfloat16)
    proj[:, d.d_in_proj:] = 0
    dy = torch.randn(B, L, d.d_inner, device="cuda").to(torch.bfloat16)
    dproj, dwB, dwC, ddtb, dD, dCb, dBb = C.m3_bwd(
        proj, dy, m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D, B, L, d.n_heads,
        m.A_floor, 1e-6)
    p32 = proj[:, :d.d_in_proj].float().clone().requires_grad_(True)
    params = [m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.D, m.C_bias, m.B_bias]
    for p in params:
        p.grad = None
    y = _oracle_y(m, p32, B, L)
    (y * dy.float()).sum().backward()
    assert rel(dproj[:, :d.d_in_proj], p32.grad) < 3e-2, rel(dproj[:, :d.d_in_proj], p32.grad)
    # column groups separately: z, x, B, C, dd_dt, dd_A, trap, angles
    sizes = [d.d_inner, d.d_inner, d.d_state, d.d_state, d.n_heads, d.n_heads, d.n_heads, d.R]
    off = 0
    for name, s in zip(["z", "x", "B", "C", "dd_dt", "dd_A", "trap", "ang"], sizes):
        e = rel(dproj[:, off:off + s], p32.grad[:, off:off + s])
        assert e < 5e-2, (name, e)
        off += s
    assert (dproj[:, d.d_in_proj:] == 0).all()
    for got, p, name in [(dwB, m.B_norm.scale, "B_norm"), (dwC, m.C_norm.scale, "C_norm"),
                         (ddtb, m.dt_bias, "dt_bias"), (dD, m.D, "D"), (dCb, m.C_bias, "C_bias"),
                         (dBb, m.B_bias, "B_bias")]:
        assert rel(got, p.grad) < 5e-2, (name, rel(got, p.grad))


def test_fused_layer_matches_torch_path():
    """Whole pre-norm half_glu1 layer: fused CUDA autograd vs the torch composition."""
    from sigma0_b200.models.mamba3 import Mamba3
    from sigma0_b200.models.layers import SequenceLayer
    torch.manual_seed(3)
    H, B, L = 256, 2, 130
    layer = SequenceLayer(Mamba3(H, impl="cuda", dtype=torch.bfloat16), H).cuda()
    ref_layer = SequenceLayer(Mamba3(H, impl="torch", dtype=torch.float32), H).cuda()
    ref_layer.load_state_dict(layer.state_dict())
    x = torch.randn(B, L, H, device="cuda")
    x1 = x.clone().requires_grad_(True)
    x2 = x.clone().requires_grad_(True)
    y1 = layer(x1)
    y2 = ref_layer(x2)
    assert rel(y1 - x, y2 - x) < 3e-2
    g = torch.randn_like(y1)
    (y1 * g).sum().backward()
    (y2 * g).sum().backward()
    assert rel(x1.grad, x2.grad) < 3e-2
    for (n, p1), (_, p2) in zip(layer.named_parameters(), ref_layer.named_parameters()):
        assert rel(p1.grad, p2.grad) < 6e-2, (n, rel(p1.grad, p2.grad))


def test_linear_ce_matches_torch():
    from sigma0_b200.ops.cross_entropy import linear_cross_entropy_mean
    torch.manual_seed(0)
    T, d, V = 1000, 128, 2112
    h = torch.randn(2, T // 2, d, device="cuda", requires_grad=True)
    Wk = (torch.randn(d, V, device="cuda") * 0.05).requires_grad_(True)
    b = (torch.randn(V, device="cuda") * 0.1).requires_grad_(True)
    lab = torch.randint(0, V, (2, T // 2), device="cuda")
    w = torch.full((2, T // 2), 1.0 / T, device="cuda")
    loss, ce = linear_cross_entropy_mean(h, Wk, b, lab, w)
    loss.backward()
    h2, W2, b2 = h.detach().clone().requires_grad_(True), Wk.detach().clone().requires_grad_(True), \
        b.detach().clone().requires_grad_(True)
    logits = h2.reshape(-1, d) @ W2 + b2
    l2 = torch.nn.functional.cross_entropy(logits, lab.reshape(-1))
    l2.backward()
    assert abs(loss.item() - l2.item()) < 2e-2 * abs(l2.item())
    assert rel(h.grad, h2.grad) < 3e-2
    assert rel(Wk.grad, W2.grad) < 3e-2
    assert rel(b.grad, b2.grad) < 3e-2


def test_flat_adam_cuda_matches_cpu():
    from sigma0_b200.train.optim import FlatAdam
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 4))
    net_c = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 4))
    net_c.load_state_dict(net.state_dict())
    net = net.cuda()
    o1 = FlatAdam(net, lr=1e-2, ssm_lr=1e-3, max_grad_norm=0.5)
    o2 = FlatAdam(net_c, lr=1e-2, ssm_lr=1e-3, max_grad_norm=0.5)
    for _ in range(3):
        x = torch.randn(8, 16)
        o1.zero_grad(); o2.zero_grad()
        net(x.cuda()).pow(2).sum().backward()
        net_c(x).pow(2).sum().backward()
        o1.step(); o2.step()
    assert (o1.flat.cpu() - o2.flat).abs().max().item() < 1e-5


def test_odd_width_book_layer_paths_match_fp32():
    """The padded bf16 paths for 503-wide book layers (mixer GEMMs and dense layers)."""
    from sigma0_b200.ops.linear import linear_bf16
    torch.manual_seed(0)
    x = torch.randn(300, 503, device="cuda", requires_grad=True)
    w = torch.randn(503, 1024, device="cuda", requires_grad=True)
    b = torch.randn(1024, device="cuda", requires_grad=True)
    y = linear_bf16(x, w, b)
    yr = x @ w + b
    assert rel(y, yr) < 1e-2
    g = torch.randn_like(y)
    gx, gw, gb = torch.autograd.grad(y, (x, w, b), g)
    rx, rw, rb = torch.autograd.grad(yr, (x, w, b), g)
    assert rel(gx, rx) < 1e-2 and rel(gw, rw) < 1e-2 and rel(gb, rb) < 1e-5
    m = _layer(H=503, seed=3)
    u = torch.randn(2, 130, 503, device="cuda") * 0.5
    y = m(u)
    m.impl = "torch"
    y2 = m(u)
    assert rel(y, y2) < 3e-2, rel(y, y2)


@pytest.mark.parametrize("T,D", [(300, 2048), (5000, 2048), (257, 1024), (100, 2048), (40, 64), (3000, 4096),
                                 (77, 4096), (500, 3072), (64, 8192)])
def test_rmsnorm_kernels_match_fp32(T, D):
    """rms_fwd / rms_bwd (register, pipelined and wide-row variants) against fp32 autograd."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    torch.manual_seed(D + T)
    x = (torch.randn(T, D, device="cuda") * 2).to(torch.bfloat16)
    w = torch.randn(D, device="cuda") * 0.5 + 1
    g = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    y, r = C.rms_fwd(x, w, 1e-6)
    xf = x.float().requires_grad_(True)
    wf = w.clone().requires_grad_(True)
    yr = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-6) * wf
    (yr * g.float()).sum().backward()
    assert rel(y, yr.detach()) < 1e-2
    dx, dw = C.rms_bwd(g, x, w, r)
    assert rel(dx, xf.grad) < 1e-2, rel(dx, xf.grad)
    assert rel(dw, wf.grad) < 1e-3, rel(dw, wf.grad)


@pytest.mark.parametrize("T,D,res", [(3000, 1024, True), (200, 1024, False), (150, 768, True), (90, 1024, True),
                                     (500, 512, True)])
def test_layernorm_backward_matches_fp32(T, D, res):
    """ln_bwd (register and pipelined variants) with the residual gradient against fp32 autograd."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    torch.manual_seed(T + D)
    x = torch.randn(T, D, device="cuda") * 2 + 0.5
    w = torch.randn(D, device="cuda") * 0.5 + 1
    b = torch.randn(D, device="cuda") * 0.1
    xn, mu, rs = C.ln_fwd(x, w, b, 1e-6)
    g = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    dres = torch.randn(T, D, device="cuda") if res else None
    xf, wf, bf = (t.clone().requires_grad_(True) for t in (x, w, b))
    yr = torch.nn.functional.layer_norm(xf, (D,), wf, bf, 1e-6)
    (yr * g.float()).sum().backward()
    dx, dw, db = C.ln_bwd(g, x, mu, rs, w, dres)
    want = xf.grad + (dres if res else 0)
    assert rel(dx, want) < 1e-3, rel(dx, want)
    assert rel(dw, wf.grad) < 1e-3 and rel(db, bf.grad) < 1e-3


@pytest.mark.parametrize("T,D", [(3000, 1024), (100, 512), (77, 1024), (50, 200)])
def test_glu_residual_backward_matches_fp32(T, D):
    """glu_res_bwd (column-owner and row variants) against fp32 autograd of x + g * sigmoid(h + b)."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    torch.manual_seed(T * 7 + D)
    g = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    h = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    b = torch.randn(D, device="cuda") * 0.3
    dout = torch.randn(T, D, device="cuda")
    gf, hf, bf = g.float().requires_grad_(True), h.float().requires_grad_(True), b.clone().requires_grad_(True)
    (((gf * torch.sigmoid(hf + bf)) * dout).sum()).backward()
    dh, dgp, db = C.glu_res_bwd(dout, g, h, b)
    assert rel(dh, hf.grad) < 1e-2, rel(dh, hf.grad)
    assert rel(dgp, gf.grad) < 1e-5, rel(dgp, gf.grad)
    assert rel(db, bf.grad) < 1e-4, rel(db, bf.grad)


@pytest.mark.parametrize("walker", [False, True])
def test_ssd_backward_with_saved_forward_tensors_matches_recompute(walker):
    """m3_bwd given the forward's passed states and prep tensors matches m3_bwd recomputing them."""
    from sigma0_b200.ops._ext import ext
    C = ext()
    C.m3_use_tc(walker)
    m = _layer(seed=4)
    B, L = 2, 333
    d = m.dims
    ldp = (d.d_in_proj + 7) // 8 * 8
    proj = (torch.randn(B * L, ldp, device="cuda") * 0.5).to(torch.bfloat16)
    dy = torch.randn(B, L, d.d_inner, device="cuda").to(torch.bfloat16)
    args = (m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D)
    try:
        out = C.m3_fwd(proj, B, L, d.n_heads, *args, m.A_floor, 1e-6, return_prep=True)
        # y, states, final state, final angle + the prep (6 tensors for the walker, 7 otherwise)
        assert len(out) == (10 if walker else 11)
        full = C.m3_bwd(proj, dy, *args, B, L, d.n_heads, m.A_floor, 1e-6)
        saved = C.m3_bwd(proj, dy, *args, B, L, d.n_heads, m.A_floor, 1e-6, saved_states=out[1],
                         saved_prep=list(out[4:]))
    finally:
        C.m3_use_tc(None)
    # equal up to the summation order of the kernels' shared-memory atomics
    for a, b in zip(full, saved):
        assert rel(a, b) < 1e-3, rel(a, b)


def test_ssd_carry_split_matches_whole_sequence():
    """A sequence run as two pieces -- the second continued from the first one's final state
    (plus the trapezoid coupling of the boundary tokens) and angle -- gives the whole
    sequence's outputs, final state and gradients (the context-parallel building block)."""
    import math
    import torch.nn.functional as F
    from sigma0_b200.ops.mamba3_layer import mamba3_ssd_carry
    from sigma0_b200.ops.reference import mamba3_ref as ref
    m, d, proj0 = _walker_args(2, 700, 512, 6)
    B, L, L1 = 2, 700, 300
    nh, P = d.n_heads, d.headdim
    g = torch.randn(B, L, d.d_inner, device="cuda")

    def run(split):
        proj = proj0.clone().requires_grad_(True)
        pv = proj.view(B, L, -1)
        if not split:
            y, fin = mamba3_ssd_carry(proj, m, B, L)
        else:
            pa, pb = pv[:, :L1].reshape(B * L1, -1).contiguous(), pv[:, L1:].reshape(B * (L - L1), -1).contiguous()
            ya, fa = mamba3_ssd_carry(pa, m, B, L1)
            z, x, Bc, Cc, dd_dt, dd_A, trap, ang = m.split_proj(pv[..., :d.d_in_proj].float())
            DT = F.softplus(dd_dt + m.dt_bias)
            tot = torch.einsum("blr,blh->bhr", torch.tanh(ang[:, :L1]) * math.pi, DT[:, :L1])
            th = tot - 2 * math.pi * torch.floor(tot / (2 * math.pi))
            Kb = m.B_norm(Bc[:, L1 - 1])[:, None, :] + m.B_bias[None]
            k_last = ref.apply_rope(Kb, torch.cos(th), torch.sin(th))
            v_last = x[:, L1 - 1].reshape(B, nh, P)
            w0 = (1.0 - torch.sigmoid(trap[:, L1])) * DT[:, L1]
            s_in = fa + w0[..., None, None] * v_last[..., :, None] * k_last[..., None, :]
            yb, fin = mamba3_ssd_carry(pb, m, B, L - L1, s_in.contiguous(), th.contiguous())
            y = torch.cat([ya, yb], 1)
        for p_ in (m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D):
            p_.grad = None
        ((y.float() * g).sum() + fin.sum() * 1e-3).backward()
        grads = [p_.grad.clone() for p_ in (m.B_norm.scale, m.C_norm.scale, m.dt_bias, m.B_bias, m.C_bias, m.D)]
        return y.detach(), fin.detach(), proj.grad.detach(), grads

    yw, fw, gw, pw = run(False)
    ys, fs, gs, ps = run(True)
    assert rel(ys, yw) < 1e-2, rel(ys, yw)
    assert rel(fs, fw) < 1e-2, rel(fs, fw)
    assert rel(gs[:, :d.d_in_proj], gw[:, :d.d_in_proj]) < 3e-2, rel(gs, gw)
    for a, b in zip(ps, pw):
        assert rel(a, b) < 3e-2, rel(a, b)
