"""Checkpoint round trip, retention, corruption fallback and params-only restore."""
import os

import numpy as np
import pytest
import torch

from sigma0_b200.ckpt import CheckpointManager, CheckpointError, remap_step


def _args(**kw):
    from sigma0_b200.models import preset_args
    return preset_args("smoke", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_messages=4, micro_bsz=2,
                       warmup_end=0.0, **kw)


def _data():
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    ds = LobWindowDataset.from_days(make_sequences(2, 5, seed=4), 4, token_mode="22tok")
    return collate([ds[i] for i in range(2)])


def _trainer(seed=0, **kw):
    from sigma0_b200.train.trainer import Trainer
    return Trainer(_args(**kw), device=torch.device("cpu"), total_steps=20, seed=seed)


def test_resume_continues_bit_exactly(tmp_path):
    batch = _data()
    a = _trainer()
    for _ in range(2):
        a.step_device(*batch)
    mgr = CheckpointManager(str(tmp_path))
    mgr.save(2, a, metrics={"loss": 1.0})
    mgr.wait()
    a.step_device(*batch)
    b = _trainer(seed=7)
    meta = mgr.restore(b)
    assert meta["step"] == 2 and b.step_idx == 2 and b.opt.step_count == 2
    b.step_device(*batch)
    assert torch.equal(a.opt.flat, b.opt.flat)
    assert torch.equal(a.opt.m, b.opt.m) and torch.equal(a.opt.v, b.opt.v)


def test_retention_and_corruption_fallback(tmp_path):
    a = _trainer()
    mgr = CheckpointManager(str(tmp_path), max_to_keep=2, keep_period=5)
    for s in (1, 2, 3, 4, 5, 6, 7):
        mgr.save(s, a, blocking=True)
    assert mgr.steps() == [5, 6, 7]   # newest two, plus multiples of keep_period
    with open(os.path.join(str(tmp_path), "7", "state", "params.f32"), "r+b") as f:
        f.seek(16)
        f.write(b"\x00\x01\x02\x03")
    assert not mgr.verify(7) and mgr.verify(6)
    meta = mgr.restore(_trainer(seed=3))
    assert meta["restored_step"] == 6
    with pytest.raises(CheckpointError):
        mgr.restore(_trainer(), step=7)


def test_params_only_restore_into_other_layout(tmp_path):
    a = _trainer()
    a.step_device(*_data())
    mgr = CheckpointManager(str(tmp_path))
    mgr.save(1, a, blocking=True)
    b = _trainer(seed=5, opt_config="noBCdecay")   # different optimizer grouping -> different flat layout
    mgr.restore(b, params_only=True)
    pa = dict(a.model.named_parameters())
    for n, p in b.model.named_parameters():
        assert torch.equal(p, pa[n]), n


def test_export_npz_uses_flax_paths(tmp_path):
    a = _trainer()
    p = os.path.join(str(tmp_path), "params.npz")
    CheckpointManager(str(tmp_path)).export_params_npz(a, p)
    z = np.load(p)
    assert "params/decoder/kernel" in z.files
    assert any(k.startswith("params/message_encoder/encoder/embedding") for k in z.files)


def test_remap_step():
    assert remap_step(100, 64, 32) == 200 and remap_step(100, 64, 64) == 100 and remap_step(7, 4, 8) == 3


def test_context_parallel_wrappers_keep_parameter_paths():
    """Wrapping blocks for context parallelism does not change the checkpoint paths."""
    import torch
    from sigma0_b200.ckpt.checkpoint import flax_path
    from sigma0_b200.models.gdn import GDN
    from sigma0_b200.models.mamba3 import Mamba3
    from sigma0_b200.models.nsa import NSABlock
    from sigma0_b200.models.transformer import TransformerBlock
    from sigma0_b200.parallel.cp import shard_model_cp

    def build():
        torch.manual_seed(0)
        return torch.nn.Sequential(Mamba3(64, d_state=16, headdim=16, chunk_size=16), TransformerBlock(64, n_heads=4),
                                   NSABlock(64, n_heads=4, block_size=8, select_block=16),
                                   GDN(64, num_heads=4, head_dim=16))
    plain = [flax_path(n) for n, _ in build().named_parameters()]
    wrapped = [flax_path(n) for n, _ in shard_model_cp(build()).named_parameters()]
    assert plain == wrapped


def test_pinned_checkpoints_detect_drift(tmp_path):
    """A pinned name fixes one step by its metadata hash: it resolves while the step is
    unchanged, and a damaged state file, a rewritten step, a removed step or (when asked) a
    newer step raise ModelStoreError."""
    import glob
    import shutil
    from sigma0_b200.pipeline.model_store import ModelStoreError, pin, resolve
    a = _trainer()
    mgr = CheckpointManager(str(tmp_path / "run"))
    mgr.save(3, a, blocking=True)
    mgr.save(6, a, blocking=True)
    store = str(tmp_path / "pins.json")
    pin(store, "bg-flow", str(tmp_path / "run"), 3, role="background_order_flow", rationale="best KS")
    e = resolve(store, "bg-flow")
    assert e["step"] == 3 and e["role"] == "background_order_flow"
    with pytest.raises(ModelStoreError):
        resolve(store, "bg-flow", require_latest=True)                  # step 6 is newer
    with pytest.raises(ModelStoreError):
        resolve(store, "signal")
    victim = sorted(glob.glob(str(tmp_path / "run" / "3" / "state" / "*")))[0]
    with open(victim, "r+b") as f:                      # a state file changed behind the pin's back
        b = f.read(1)
        f.seek(0)
        f.write(bytes([b[0] ^ 0xFF]))
    with pytest.raises(ModelStoreError):
        resolve(store, "bg-flow")
    mgr.save(3, a, metrics={"loss": 2.0}, blocking=True)   # saved again with other contents
    with pytest.raises(ModelStoreError):
        resolve(store, "bg-flow")
    pin(store, "sig", str(tmp_path / "run"), 6)
    shutil.rmtree(str(tmp_path / "run" / "6"))
    with pytest.raises(ModelStoreError):
        resolve(store, "sig")


def test_checkpoint_inspector(tmp_path, capsys):
    """The inspector summarises native and Orbax steps (layout, leaves and parameter counts per
    top-level key, integrity, sampled arrays) and exits non-zero on a damaged step."""
    import glob
    import json
    from sigma0_b200.ckpt.inspect import main, summarize
    a = _trainer()
    n_params = sum(p.numel() for p in a.model.parameters())
    CheckpointManager(str(tmp_path / "nat")).save(2, a, config={"d_model": 64, "architecture": "mamba3"},
                                                  blocking=True)
    s = summarize(str(tmp_path / "nat"), sample_arrays=2)
    assert s["layout"] == "native" and s["intact"] and s["step"] == 2 and s["d_model"] == 64
    assert s["elements"]["params"] == n_params and len(s["samples"]) == 2 and s["samples"][0]["finite"]
    CheckpointManager(str(tmp_path / "orb"), fmt="orbax").save(4, a, config={"d_model": 64}, blocking=True)
    s = summarize(str(tmp_path / "orb" / "4"), sample_arrays=1)
    assert s["layout"] == "orbax" and s["intact"] and s["elements"]["params"] == n_params
    assert main([str(tmp_path / "orb"), "--json"]) == 0 and json.loads(capsys.readouterr().out)["step"] == 4
    victim = sorted(glob.glob(str(tmp_path / "nat" / "2" / "state" / "*.f32")))[0]
    with open(victim, "r+b") as f:
        f.write(b"\xff\xff\xff\xff")
    assert main([str(tmp_path / "nat")]) == 1
