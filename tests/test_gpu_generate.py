"""GPU numerics of the decode, engine and generation kernels against CPU oracles."""
import numpy as np
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
        m.in_proj.kernel.mul_(2.0)
    return m


def test_decode_step_and_prefill_match_oracle():
    """CUDA prefill (chunked, with final state) + CUDA decode steps == fp32 recurrence."""
    from sigma0_b200.ops.reference import mamba3_ref as ref
    m = _layer()
    B, L, S = 3, 150, 6
    u = torch.randn(B, L + S, 512, device="cuda") * 0.5
    with torch.no_grad():
        st, yp = m.prefill(u[:, :L])
        outs = [yp]
        for t in range(S):
            st, y = m.step(st, u[:, L + t:L + t + 1])
            outs.append(y)
        got = torch.cat(outs, 1)
        m.impl = "torch"
        want = m(u.double().float())
    assert rel(got, want) < 3e-2, rel(got, want)
    assert rel(got[:, L:], want[:, L:]) < 3e-2


@pytest.mark.parametrize("T", [2, 5, 8])
def test_multi_token_decode_matches_single_steps(T):
    """One T-token recurrent step (state read/written once) == T one-token steps,
    including the carried angle, key and value; odd head counts cover a partial
    head group."""
    for H in (512, 448):
        m = _layer(H, seed=T)
        B, L = 4, 70
        u = torch.randn(B, L + T, H, device="cuda") * 0.5
        with torch.no_grad():
            st1, _ = m.prefill(u[:, :L])
            st2 = tuple(s.clone() for s in st1)
            ys = []
            for t in range(T):
                st1, y = m.step(st1, u[:, L + t:L + t + 1])
                ys.append(y)
            st2, y2 = m.step(st2, u[:, L:L + T])
        y1 = torch.cat(ys, 1)
        assert rel(y2, y1) < 1e-2, rel(y2, y1)
        for a, b in zip(st2, st1):
            assert rel(a, b) < 1e-4, rel(a, b)


def _rand_engine_stream(n_books, n_msgs, seed):
    from sigma0_b200.data.synthetic import generate_day
    days = [generate_day(n_msgs, seed=seed + i) for i in range(n_books)]
    return days


def test_engine_kernel_matches_cpu_orderbook():
    from sigma0_b200.engine.book import EngineConfig, init_msgs_from_l2, book_from_l2
    from sigma0_b200.engine.batched import BatchedEngine
    cfg = EngineConfig()
    days = _rand_engine_stream(9, 300, 11)
    eng = BatchedEngine(9, cfg, device="cuda")
    init = np.stack([init_msgs_from_l2(d.l2_init, cfg) for d in days])
    eng.process(init)
    msgs = np.stack([d.engine_msgs for d in days])
    # perturb a few messages so cancels miss and fall back
    msgs[:, ::37, 4] = 123456789
    for k0 in range(0, 300, 100):
        eng.process(msgs[:, k0:k0 + 100])
    asks, bids = eng.sides()
    l2 = eng.l2(10).cpu().numpy()
    tr = eng.trade_rows()
    for b, d in enumerate(days):
        ob = book_from_l2(d.l2_init, cfg)
        ob.process_many(msgs[b])
        assert np.array_equal(ob.asks, asks[b]), b
        assert np.array_equal(ob.bids, bids[b]), b
        assert np.array_equal(ob.trades, tr[b]), b
        assert np.array_equal(ob.l2(10), l2[b]), b


def test_gen_apply_matches_cpu_oracle():
    """Decode + order-id resolution + match + L2 + book image, message by message."""
    from sigma0_b200.ops._ext import ext
    from sigma0_b200.encoding import get_tokenizer
    from sigma0_b200.engine.book import EngineConfig, init_msgs_from_l2, book_from_l2
    from sigma0_b200.infer.generate import apply_message_cpu, gen_layout, safe_mid_price, _best_quotes
    tok = get_tokenizer("22tok")
    cfg = EngineConfig()
    nb, n = 6, 120
    days = _rand_engine_stream(nb, n, 40)
    obs = [book_from_l2(d.l2_init, cfg) for d in days]
    asks = torch.full((nb, cfg.n_orders, 6), -1, dtype=torch.int32, device="cuda")
    bids = torch.full_like(asks, -1)
    trades = torch.full((nb, cfg.n_trades, 8), -1, dtype=torch.int32, device="cuda")
    init = torch.from_numpy(np.stack([init_msgs_from_l2(d.l2_init, cfg) for d in days]).astype(np.int32)).cuda()
    ext().eng_process(asks, bids, trades, init, cfg.init_id, cfg.book_depth, cfg.cancel_mode,
                      cfg.type_4_interpretation, cfg.check_book_fill)
    pm = [safe_mid_price(*_best_quotes(ob), 100) for ob in obs]
    p_mid = torch.tensor(pm, dtype=torch.int32, device="cuda")
    lay = gen_layout(tok, 100, 500, 10)
    o_raw = torch.zeros(nb, 14, dtype=torch.int32, device="cuda")
    o_msg = torch.zeros(nb, 8, dtype=torch.int32, device="cuda")
    o_prov = torch.zeros(nb, dtype=torch.int32, device="cuda")
    o_l2 = torch.zeros(nb, 40, dtype=torch.int32, device="cuda")
    img = torch.zeros(nb, 503, dtype=torch.float32, device="cuda")
    oid = torch.zeros(1, dtype=torch.int32, device="cuda")
    tin = torch.zeros(nb, 2, dtype=torch.int32, device="cuda")
    toks_all = np.stack([tok.encode_msgs(d.msgs) for d in days])
    provs = set()
    for k in range(n):
        oid.fill_(n - k)
        t = torch.from_numpy(toks_all[:, k].astype(np.int64)).cuda()
        inj = [1, 1 + (k % 2) * 3, k % 2, 55, -1 - k % 3] if k % 17 == 5 else None   # do(Q) at a few steps
        ext().gen_apply(asks, bids, trades, t, lay, cfg.init_id, cfg.book_depth, cfg.cancel_mode,
                        cfg.type_4_interpretation, cfg.check_book_fill, oid, p_mid, tin, o_raw, o_msg, o_prov, o_l2,
                        img, True, torch.tensor(inj, dtype=torch.int32, device="cuda") if inj else None)
        for b in range(nb):
            raw, msg, prov, l2, im, pmn = apply_message_cpu(obs[b], toks_all[b, k], tok, pm[b], n - k, inject=inj)
            pm[b] = pmn
            provs.add(prov)
            assert np.array_equal(o_raw[b].cpu().numpy(), raw), (k, b, o_raw[b], raw)
            assert np.array_equal(o_msg[b].cpu().numpy(), msg), (k, b)
            assert o_prov[b].item() == prov, (k, b)
            assert np.array_equal(o_l2[b].cpu().numpy(), l2), (k, b)
            assert p_mid[b].item() == pmn
            np.testing.assert_allclose(img[b].cpu().numpy(), im, rtol=1e-6, atol=1e-6)
    assert len(provs) >= 2   # new orders and resolved cancels both exercised


def test_gen_sample_argmax_and_gumbel():
    from sigma0_b200.ops._ext import ext
    torch.manual_seed(0)
    B, V = 64, 12288
    logits = torch.randn(B, V, device="cuda")
    bias = torch.randn(V, device="cuda") * 0.1
    allow = (torch.rand(V, device="cuda") < 0.3).to(torch.uint8)
    ctr = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = torch.zeros(B, 3, dtype=torch.int64, device="cuda")
    ext().gen_sample(logits, bias, allow, 7, ctr, 0, 1, out, 1, 3)
    ref = (logits + bias).masked_fill(allow == 0, float("-inf")).argmax(-1)
    assert torch.equal(out[:, 1], ref)
    # Gumbel-max frequencies on a small support match the softmax
    V2, R = 8, 4096
    lg = torch.tensor([0.0, 1.0, -1.0, 0.5, 2.0, -3.0, 0.0, 1.5], device="cuda").repeat(R, 1)
    al = torch.ones(V2, dtype=torch.uint8, device="cuda")
    al[5] = 0
    cnt = torch.zeros(V2, device="cuda")
    o2 = torch.zeros(R, dtype=torch.int64, device="cuda")
    for i in range(16):
        ctr.fill_(i)
        ext().gen_sample(lg, None, al, 3, ctr, 5, -1, o2, 0, 1)
        cnt += torch.bincount(o2, minlength=V2).float()
    p = torch.softmax(lg[0].masked_fill(al == 0, float("-inf")), 0)
    freq = cnt / cnt.sum()
    assert cnt[5].item() == 0
    assert (freq - p).abs().max().item() < 0.01, (freq, p)


def test_gen_time_tokens_matches_cpu():
    from sigma0_b200.ops._ext import ext
    from sigma0_b200.encoding import get_tokenizer
    from sigma0_b200.infer.generate import time_tokens_cpu
    tok = get_tokenizer("22tok")
    off = tok.vocab.codes["time"].offset
    B = 300
    g = torch.Generator().manual_seed(0)
    msg = torch.randint(off, off + 1000, (B, tok.MSG_LEN), generator=g)
    time = torch.stack([torch.randint(34200, 57600, (B,), generator=g),
                        torch.randint(0, 10**9, (B,), generator=g)], 1).int()
    m1, t1 = msg.clone(), time.clone()
    time_tokens_cpu(m1, tok, t1)
    m2, t2 = msg.cuda(), time.cuda()
    ext().gen_time_tokens(m2, tok.FIELD_START["delta_t_s"], off, t2)
    assert torch.equal(m2.cpu(), m1) and torch.equal(t2.cpu(), t1)


def test_generator_graph_equals_eager():
    """A CUDA-graph replay of a whole message produces exactly the eager tokens."""
    from sigma0_b200.data.synthetic import make_sequences
    from sigma0_b200.data.book_transform import transform_books_numpy
    from sigma0_b200.encoding import get_tokenizer, START_TOK
    from sigma0_b200.infer import Generator
    from sigma0_b200.models import preset_args, build_model
    torch.manual_seed(0)
    a = preset_args("350m", n_layers=2, n_messages=12, impl="cuda")
    m = build_model(a).cuda().eval()
    tok = get_tokenizer("22tok")
    days = make_sequences(4, 16, seed=2)
    x, bk, last, l2s, em = [], [], [], [], []
    for d in days:
        t = tok.encode_msgs(d.msgs[:12]).reshape(-1)
        x.append(np.concatenate([[START_TOK], t[:-1]]))
        last.append(t[-1])
        bk.append(transform_books_numpy(d.books[:12]))
        l2s.append(d.l2_init)
        em.append(d.engine_msgs[:12])
    ctx = (torch.tensor(np.stack(x)), torch.tensor(np.stack(bk)), torch.tensor(last), np.stack(l2s), np.stack(em))
    outs = []
    for graphs in (False, True):
        g = Generator(m, "22tok", top_n=-1, seed=5, use_graphs=graphs)
        g.condition(*ctx)
        outs.append(g.generate(4))
    assert torch.equal(outs[0].tokens, outs[1].tokens)
    assert torch.equal(outs[0].l2, outs[1].l2)
    # the engine path agrees with the CPU engine replaying the emitted messages
    from sigma0_b200.engine.book import EngineConfig, book_from_l2
    raw = outs[1].raw.cpu().numpy().astype(np.int64)
    for b in range(4):
        ob = book_from_l2(l2s[b], EngineConfig())
        ob.process_many(em[b])
        for k in range(4):
            r = raw[b, k]
            ob.process(np.array([r[1], r[2] * 2 - 1, r[5], r[3], r[0], -88, r[8], r[9]]))
            assert np.array_equal(ob.l2(10), outs[1].l2[b, k].cpu().numpy())


def test_fused_layer_prefill_matches_forward_and_steps():
    """SequenceLayer.prefill on the fused CUDA path: output == the training forward, and the
    returned state continues like stepping the unfused layer token by token."""
    from sigma0_b200.models.layers import SequenceLayer
    from sigma0_b200.models.mamba3 import Mamba3
    torch.manual_seed(3)
    H = 256
    layer = SequenceLayer(Mamba3(H, impl="cuda"), H, "half_glu1", True, 0.0).cuda()
    with torch.no_grad():
        layer.seq.B_bias.normal_(0, 0.5)
        layer.seq.C_bias.normal_(0, 0.5)
        layer.out2.kernel.mul_(2.0)
    x = torch.randn(2, 130, H, device="cuda")
    with torch.no_grad():
        want = layer(x)
        st, got = layer.prefill(x[:, :128])
        assert rel(got, want[:, :128]) < 1e-2, rel(got, want[:, :128])
        for t in (128, 129):
            st, y = layer.step(st, x[:, t:t + 1])
            assert rel(y, want[:, t:t + 1]) < 3e-2, (t, rel(y, want[:, t:t + 1]))
