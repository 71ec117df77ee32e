"""Muon, legacy-norm epsilons and the ES low-rank fold."""
import os

import pytest
import torch


def _args(**kw):
    from sigma0_b200.models import preset_args
    return preset_args("smoke", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_messages=4, micro_bsz=2,
                       warmup_end=0.0, **kw)


def _batch():
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    ds = LobWindowDataset.from_days(make_sequences(2, 5, seed=4), 4, token_mode="22tok")
    return collate([ds[0], ds[1]])


def test_newton_schulz_orthogonalizes():
    from sigma0_b200.train.muon import orthogonalize
    torch.manual_seed(0)
    for shape in ((64, 32), (32, 96)):
        G = torch.randn(*shape)
        s = torch.linalg.svdvals(orthogonalize(G))
        assert s.min() > 0.5 and s.max() < 1.5, s


def test_muon_training_step():
    from sigma0_b200.train.trainer import Trainer
    tr = Trainer(_args(opt_config="muon"), device=torch.device("cpu"), total_steps=20, seed=0)
    b = _batch()
    l0 = float(tr.step_device(*b))
    for _ in range(6):
        l = float(tr.step_device(*b))
    assert l < l0
    o = tr.opt
    assert o.muon_names and all(torch.count_nonzero(o.m[slice(*o.slices[n])]) == 0 for n in o.muon_names)


def test_legacy_norm_epsilons(monkeypatch):
    from sigma0_b200.models import build_model
    from sigma0_b200.models.mamba3 import Mamba3
    torch.manual_seed(0)
    a = build_model(_args())
    monkeypatch.setenv("MAMBA3_LEGACY_NORM", "1")
    torch.manual_seed(0)
    b = build_model(_args())
    ma = [m for m in a.modules() if isinstance(m, Mamba3)][0]
    mb = [m for m in b.modules() if isinstance(m, Mamba3)][0]
    assert ma.B_norm.eps == 1e-6 and mb.B_norm.eps == mb.dims.d_state and mb.out_norm.eps == mb.dims.d_inner
    tok, lab, book = _batch()
    with torch.no_grad():
        assert not torch.allclose(a(tok, book), b(tok, book))


def test_es_fold_zero_sigma_is_exact_and_hooks_clean_up():
    from sigma0_b200.models import build_model
    from sigma0_b200.models.es_fold import sample_factors, es_perturbation, fold_kernel
    torch.manual_seed(0)
    m = build_model(_args()).eval()
    tok, lab, book = _batch()
    with torch.no_grad():
        base = m(tok, book)
        f0 = sample_factors(m, rank=4, sigma=0.0, seed=1)
        assert f0 and all(torch.count_nonzero(v["A"]) == 0 for v in f0.values())
        with es_perturbation(m, f0):
            assert torch.equal(m(tok, book), base)
        f1 = sample_factors(m, rank=4, sigma=0.1, seed=1)
        with es_perturbation(m, f1):
            pert = m(tok, book)
        assert not torch.allclose(pert, base)
        assert torch.equal(m(tok, book), base)          # hooks removed
        name = next(iter(f1))
        dense = dict(m.named_modules())[name]
        x = torch.randn(3, dense.d_in)
        with es_perturbation(m, {name: f1[name]}):
            hooked = dense(x)
        assert torch.allclose(hooked, fold_kernel(f1, name, x, dense(x)), atol=1e-6)
