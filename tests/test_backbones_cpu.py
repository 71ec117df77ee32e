"""Every backbone builds under the registry, runs forward/backward inside the LOB
model, and its recurrent decode matches its training forward."""
import pytest
import torch

from sigma0_b200.models import preset_args, build_model, build_backbone
from sigma0_b200.models.gdn import GDN, gated_delta_chunked, gated_delta_recurrent
from sigma0_b200.models.transformer import TransformerBlock
from sigma0_b200.models.nsa import NSABlock
from sigma0_b200.models.s5 import make_s5_factory
from sigma0_b200.encoding import set_token_mode


@pytest.mark.parametrize("kda", [False, True])
def test_gdn_chunked_equals_recurrent(kda):
    torch.manual_seed(0)
    B, L, nh, hd, hvd = 2, 37, 2, 8, 16
    q = torch.randn(B, L, nh, hd) * 0.3
    k = torch.nn.functional.normalize(torch.randn(B, L, nh, hd), dim=-1)
    v = torch.randn(B, L, nh, hvd)
    beta = torch.rand(B, L, nh)
    alog = torch.nn.functional.logsigmoid(torch.randn(B, L, nh, hd if kda else 1) + 2)
    o1, S1 = gated_delta_chunked(q, k, v, beta, alog, chunk=8)
    o2, S2 = gated_delta_recurrent(q, k, v, beta, alog)
    assert (o1 - o2).abs().max() < 1e-4
    assert (S1 - S2).abs().max() < 1e-4


@pytest.mark.parametrize("arch", ["mamba3", "gdn", "kda", "s5", "transformer", "nsa", "hybrid_mamba3"])
def test_backbone_in_lob_model(arch):
    torch.manual_seed(0)
    set_token_mode("22tok")
    a = preset_args("smoke", architecture=arch, d_model=64, vocab_size=64, d_book=16, n_book_pre_layers=1,
                    n_layers=4, n_heads=4, gdn_head_dim=16, ssm_size_base=16, blocks=2, block_size=22,
                    hybrid_attn_heads=4, mamba3_d_state=16, mamba3_headdim=16)
    m = build_model(a)
    B, L = 2, 44
    tok = torch.randint(0, 64, (B, L))
    book = torch.randn(B, 2, 16)
    lab = torch.randint(0, 64, (B, L))
    loss, _ = m.loss(tok, book, lab)
    loss.backward()
    assert torch.isfinite(loss)
    grads = [p.grad for p in m.parameters() if p.grad is not None]
    assert len(grads) > 0.8 * len(list(m.parameters()))


def test_transformer_decode_matches_forward():
    torch.manual_seed(0)
    blk = TransformerBlock(32, n_heads=4, max_cache_len=64)
    x = torch.randn(2, 20, 32)
    full = blk(x)
    st = blk.initial_state(2)
    outs = []
    for t in range(20):
        st, y = blk.step(st, x[:, t:t + 1])
        outs.append(y)
    assert (torch.cat(outs, 1) - full).abs().max() < 1e-4
    st2, out2 = blk.prefill(x[:, :12])
    st2, y = blk.step(st2, x[:, 12:13])
    assert (y - full[:, 12:13]).abs().max() < 1e-4


def test_gdn_layer_decode_matches_forward():
    torch.manual_seed(0)
    for kda in (False, True):
        m = GDN(32, num_heads=2, head_dim=16, chunk_size=8, use_kda=kda)
        x = torch.randn(2, 19, 32)
        full = m(x)
        st = m.initial_state(2)
        outs = []
        for t in range(19):
            st, y = m.step(st, x[:, t:t + 1])
            outs.append(y)
        assert (torch.cat(outs, 1) - full).abs().max() < 1e-4


def test_s5_decode_matches_forward():
    torch.manual_seed(0)
    m = make_s5_factory(16, 2)(24)
    x = torch.randn(2, 70, 24)
    full = m(x)
    st = m.initial_state(2)
    outs = []
    for s in range(0, 70, 10):
        st, y = m.step(st, x[:, s:s + 10])
        outs.append(y)
    assert (torch.cat(outs, 1) - full).abs().max() < 1e-4


def test_nsa_reference_mode_runs():
    torch.manual_seed(0)
    blk = NSABlock(32, n_heads=4, block_size=4, block_counts=2)
    x = torch.randn(2, 24, 32, requires_grad=True)
    y = blk(x)
    y.sum().backward()
    assert y.shape == x.shape and torch.isfinite(x.grad).all()
    blk2 = NSABlock(32, n_heads=4, block_size=4, select_block=8, block_counts=2, window_size=6,
                    full_causal_window=False)
    assert blk2(x).shape == x.shape
