"""Head-parallel GDN / KDA mixer and transformer block on CPU ranks (gloo, world 2)
against the single-process modules: outputs, input gradients, and the gradient of every
parameter slice (replicated parameters receive the full gradient on every rank), and the
consolidated state (``full_state_dict``) against the single-device block's parameters."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rel(a, b):
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _module(kind):
    torch.manual_seed(0)
    if kind in ("gdn", "kda"):
        from sigma0_b200.models.gdn import GDN
        m = GDN(64, num_heads=4, head_dim=16, expand_v=2, chunk_size=16, use_kda=kind == "kda")
        with torch.no_grad():
            m.out_norm.scale.normal_(1.0, 0.3)
    elif kind.startswith("nsa"):
        from sigma0_b200.models.nsa import NSABlock
        m = NSABlock(64, n_heads=4, d_ff=128, block_size=8, select_block=16, block_counts=2, window_size=20,
                     full_causal_window=kind == "nsa", pe_type="rope" if kind == "nsa" else "sinusoidal")
    else:
        from sigma0_b200.models.transformer import TransformerBlock
        m = TransformerBlock(64, n_heads=4, d_ff=128)
        with torch.no_grad():
            for p in m.parameters():
                if p.dim() == 1 or (p.dim() == 2 and p.shape[0] <= 4):
                    p.normal_(0, 0.2)
    return m


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randn(2, 40, 64, generator=g), torch.randn(2, 40, 64, generator=g)


def _worker(rank, world, port, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=120))
    try:
        torch.set_num_threads(1)
        from sigma0_b200.parallel.tp_heads import GDNTP, NSABlockTP, TransformerBlockTP
        full = _module(kind)
        m = (GDNTP(full, None) if kind in ("gdn", "kda") else
             NSABlockTP(full, None) if kind.startswith("nsa") else TransformerBlockTP(full, None))
        u, gout = _data()
        u.requires_grad_(True)
        y = m(u)
        (y * gout).sum().backward()
        torch.save({"y": y.detach(), "du": u.grad, "full_sd": m.full_state_dict(), "grads": {n: p.grad for n, p in m.named_parameters()},
                    "h0": m.h0, "nhl": m.nhl, "f0": getattr(m, "f0", 0), "fl": getattr(m, "fl", 0)},
                   f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["gdn", "kda", "transformer", "nsa", "nsa_window"])
def test_head_parallel_matches_full(kind, tmp_path):
    full = _module(kind)
    u, gout = _data()
    u.requires_grad_(True)
    y = full(u)
    (y * gout).sum().backward()
    out = str(tmp_path / "r")
    mp.spawn(_worker, args=(2, _port(), kind, out), nprocs=2, join=True)
    res = [torch.load(f"{out}.{r}") for r in range(2)]
    for r in res:
        assert _rel(r["y"], y.detach()) < 2e-5 and _rel(r["du"], u.grad) < 2e-5
        g, h0, n = r["grads"], r["h0"], r["nhl"]
        if kind in ("gdn", "kda"):
            hd, hvd = full.hd, full.hvd
            checks = [("q_w", full.q_proj.kernel.grad[:, h0 * hd:(h0 + n) * hd]),
                      ("v_w", full.v_proj.kernel.grad[:, h0 * hvd:(h0 + n) * hvd]),
                      ("b_b", full.b_proj.bias.grad[h0:h0 + n]),
                      ("qc_w", full.q_conv.kernel.grad[:, h0 * hd:(h0 + n) * hd]),
                      ("o_w", full.o_proj.kernel.grad[h0 * hvd:(h0 + n) * hvd]),
                      ("out_norm_scale", full.out_norm.scale.grad), ("D", full.D.grad)]
        elif kind.startswith("nsa"):
            f0, fl, hd = r["f0"], r["fl"], full.hd
            checks = [("wq", full.q_proj.kernel.grad[:, h0 * hd:(h0 + n) * hd]),
                      ("wg", full.g_proj.kernel.grad[:, h0 * 3:(h0 + n) * 3]),
                      ("wo", full.o_proj.kernel.grad[h0 * hd:(h0 + n) * hd]),
                      ("norm1.scale", full.norm1.scale.grad), ("w1", full.ff.layers_0.kernel.grad[:, f0:f0 + fl]),
                      ("b2", full.ff.layers_2.bias.grad)]
        else:
            f0, fl, a = r["f0"], r["fl"], full.attn
            checks = [("wq", a.query.kernel.grad[:, h0:h0 + n]), ("bv", a.value.bias.grad[h0:h0 + n]),
                      ("wo", a.out.kernel.grad[h0:h0 + n].reshape(-1, 64)), ("bo", a.out.bias.grad),
                      ("norm1.scale", full.norm1.scale.grad), ("w1", full.ff.layers_0.kernel.grad[:, f0:f0 + fl]),
                      ("w2", full.ff.layers_2.kernel.grad[f0:f0 + fl]), ("b2", full.ff.layers_2.bias.grad)]
        for name, ref in checks:
            err = (g[name] - ref).norm().item()
            assert err <= 5e-5 * ref.norm().item() + 1e-6, (kind, name, err)
        # consolidation: every rank rebuilds the single-device block's parameters exactly
        sd = {n: p.detach() for n, p in full.named_parameters()}
        assert set(r["full_sd"]) == set(sd), (kind, set(sd) ^ set(r["full_sd"]))
        for name, ref in sd.items():
            assert r["full_sd"][name].shape == ref.shape and torch.equal(r["full_sd"][name], ref), (kind, name)
