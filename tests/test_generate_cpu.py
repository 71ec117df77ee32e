"""Generator on CPU: syntax, computed time tokens, engine consistency."""
import numpy as np
import torch

from sigma0_b200.data.synthetic import make_sequences
from sigma0_b200.data.book_transform import transform_books_numpy
from sigma0_b200.encoding import get_tokenizer, START_TOK
from sigma0_b200.engine.book import EngineConfig, book_from_l2
from sigma0_b200.infer import Generator, syntax_validation_matrix
from sigma0_b200.models import preset_args, build_model


def _context(days, n_ctx, tok):
    x, bk, last, l2s, em = [], [], [], [], []
    for d in days:
        t = tok.encode_msgs(d.msgs[:n_ctx]).reshape(-1)
        x.append(np.concatenate([[START_TOK], t[:-1]]))
        last.append(t[-1])
        bk.append(transform_books_numpy(d.books[:n_ctx]))
        l2s.append(d.l2_init)
        em.append(d.engine_msgs[:n_ctx])
    return (torch.tensor(np.stack(x)), torch.tensor(np.stack(bk)), torch.tensor(last), np.stack(l2s), np.stack(em))


def test_generator_cpu_syntax_time_and_engine():
    torch.manual_seed(0)
    a = preset_args("smoke", n_messages=6)
    m = build_model(a).eval()
    tok = get_tokenizer("22tok")
    days = make_sequences(2, 8, seed=3)
    x, bk, last, l2s, em = _context(days, 6, tok)
    g = Generator(m, "22tok", EngineConfig(), top_n=-1, seed=1)
    g.condition(x, bk, last, l2s, em)
    t0 = g.time.clone()
    out = g.generate(3)
    toks = out.tokens.numpy()
    allow = syntax_validation_matrix(tok, vocab_size=a.vocab_size)
    L = tok.MSG_LEN
    for b in range(2):
        for k in range(3):
            for p in range(L):
                if tok.TIME_START_I <= p <= tok.TIME_END_I:
                    continue
                assert allow[p, toks[b, k, p]], (b, k, p, toks[b, k, p])
    # absolute times advance by the sampled delta-t
    raw = out.raw.numpy().astype(np.int64)
    prev = t0.numpy().astype(np.int64)
    for k in range(3):
        ns = prev[:, 1] + raw[:, k, 7]
        s = prev[:, 0] + raw[:, k, 6] + ns // 10**9
        assert np.array_equal(raw[:, k, 8], s) and np.array_equal(raw[:, k, 9], ns % 10**9)
        prev = np.stack([raw[:, k, 8], raw[:, k, 9]], 1)
    # replaying the emitted engine messages reproduces the L2 path
    for b in range(2):
        ob = book_from_l2(l2s[b], EngineConfig(), (34200, 0))
        ob.process_many(em[b])
        for k in range(3):
            r = raw[b, k]
            ob.process(np.array([r[1], r[2] * 2 - 1, r[5], r[3], r[0], -88, r[8], r[9]]))
            assert np.array_equal(ob.l2(10), out.l2[b, k].numpy())


def test_argmax_generation_is_deterministic():
    torch.manual_seed(0)
    a = preset_args("smoke", n_messages=4)
    m = build_model(a).eval()
    tok = get_tokenizer("22tok")
    days = make_sequences(1, 6, seed=5)
    ctx = _context(days, 4, tok)
    outs = []
    for _ in range(2):
        g = Generator(m, "22tok", top_n=1)
        g.condition(*ctx)
        outs.append(g.generate(2).tokens)
    assert torch.equal(outs[0], outs[1])


def test_do_q_injection_replaces_the_order():
    torch.manual_seed(0)
    a = preset_args("smoke", n_messages=6)
    m = build_model(a).eval()
    tok = get_tokenizer("22tok")
    days = make_sequences(2, 8, seed=3)
    ctx = _context(days, 6, tok)
    g = Generator(m, "22tok", top_n=1, seed=1)
    g.condition(*ctx)
    base = g.generate(3)
    g.condition(*ctx)
    out = g.generate(3, inject={"step": 1, "event_type": 1, "side": 1, "qty": 777, "offset_ticks": -1})
    em = out.engine_msgs.numpy()
    mid_before = out.mid[:, 0].numpy()
    for b in range(2):
        assert list(em[b, 1, :4]) == [1, 1, 777, int(mid_before[b]) - 100]
        assert em[b, 1, 4] == 2            # the running new-order id at step 1 of 3
        assert out.provenance[b, 1] & 16 and not out.provenance[b, 0] & 16
    # the step before the injection is untouched
    assert torch.equal(base.tokens[:, 0], out.tokens[:, 0])
