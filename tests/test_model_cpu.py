"""Model structure, registry contract and the torch reference numerics on CPU."""
import math
from types import SimpleNamespace

import pytest
import torch

from sigma0_b200.models import (preset_args, build_model, resolve_architecture, nemotron_attention_indices,
                                available_architectures)
from sigma0_b200.ops.reference import mamba3_ref as ref
from sigma0_b200.encoding import set_token_mode


def test_75m_param_count_matches_reference():
    m = build_model(preset_args("75m"))
    n = sum(p.numel() for p in m.parameters())
    assert abs(n / 1e6 - 78.5) < 0.1   # reference: "Mamba3 d1024 x6 (78.5M, 75m)"


def test_param_tree_names():
    m = build_model(preset_args("smoke"))
    names = {n for n, _ in m.named_parameters()}
    for n in ["message_encoder.encoder.embedding", "message_encoder.layers_0.seq.in_proj.kernel",
              "message_encoder.layers_0.seq.dt_bias", "message_encoder.layers_0.seq.B_norm.scale",
              "message_encoder.layers_0.seq.out_norm.scale", "message_encoder.layers_0.seq.out_proj.kernel",
              "message_encoder.layers_0.out2.kernel", "message_encoder.layers_0.norm.scale",
              "book_encoder.projection.kernel", "fused_s5.encoder.kernel", "decoder.kernel"]:
        assert n in names, n


def test_chunked_equals_recurrent():
    torch.manual_seed(0)
    Bt, L, H, N, P, R = 2, 70, 3, 16, 8, 4
    d = torch.float64
    Q, K = torch.randn(Bt, L, H, N, dtype=d), torch.randn(Bt, L, H, N, dtype=d)
    V, Z = torch.randn(Bt, L, H, P, dtype=d), torch.randn(Bt, L, H, P, dtype=d)
    DT = torch.rand(Bt, H, L, dtype=d) * 0.1
    ADT = -torch.rand(Bt, H, L, dtype=d) * 0.1
    Tr, an = torch.randn(Bt, H, L, dtype=d), torch.randn(Bt, L, R, dtype=d)
    qb, kb, D = torch.randn(H, N, dtype=d), torch.randn(H, N, dtype=d), torch.randn(H, dtype=d)
    y1 = ref.mamba3_ssd_chunked(Q, K, V, ADT, DT, Tr, an, qb, kb, D, Z, chunk_size=16)
    y2, _ = ref.mamba3_recurrent(Q, K, V, ADT, DT, Tr, an, qb, kb, D, Z)
    assert (y1 - y2).abs().max().item() < 1e-10


def test_model_step_matches_forward():
    """Recurrent decode of the whole LOB model equals the training forward."""
    torch.manual_seed(0)
    a = preset_args("smoke", d_model=64, mamba3_d_state=16, mamba3_headdim=16, vocab_size=64,
                    n_book_pre_layers=1, d_book=16, use_book_data=True)
    set_token_mode("22tok")
    m = build_model(a)
    B, L = 2, 44
    tok = torch.randint(0, 64, (B, L))
    book = torch.randn(B, L // 22, 16)
    full = m(tok, book)
    st = m.initial_state(B)
    outs = []
    bk = m.repeat_book(book, L)
    for t in range(L):
        st, lp = m.step(st, tok[:, t:t + 1], bk[:, t:t + 1])
        outs.append(lp)
    step = torch.cat(outs, 1)
    assert (full - step).abs().max().item() < 2e-4


def test_registry_contract():
    assert available_architectures()[0] == "mamba3"
    assert resolve_architecture() == "mamba3"
    assert resolve_architecture("gdn") == "gdn"
    assert resolve_architecture(model_type="transformer", ssm_type="s5") == "transformer"
    with pytest.raises(ValueError):
        resolve_architecture("gdn", ssm_type="kda")
    with pytest.raises(ValueError):
        resolve_architecture("mamba2")
    assert nemotron_attention_indices(31) == (8, 13, 17, 22)
    assert nemotron_attention_indices(12) == (3, 9)


def test_cpu_training_reduces_loss():
    from sigma0_b200.train.trainer import Trainer
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    a = preset_args("smoke", ssm_lr_base=3e-3, warmup_end=0.0)
    tr = Trainer(a, device=torch.device("cpu"), total_steps=100)
    days = make_sequences(2, 21, seed=0)
    ds = LobWindowDataset.from_days(days, 20, token_mode=a.token_mode)
    batch = collate([ds[0], ds[1]])
    l0 = tr.train_step(batch)
    for _ in range(9):
        l = tr.train_step(batch)
    assert l < l0 - 0.5, (l0, l)
