"""Orbax StandardSave layout (zarr v2 arrays under Flax key paths) without Orbax: a model
round-trips bit-exact through CheckpointManager(fmt="orbax"); a hand-built step directory
in the documented layout (several chunks, zlib, a missing fill-value chunk, bfloat16, the
reference's extra items) restores into a LobModel; OCDBT and blosc are refused clearly."""
import json
import os
import zlib

import numpy as np
import pytest
import torch

from sigma0_b200.ckpt import CheckpointManager, OrbaxFormatError, read_standard_item
from sigma0_b200.ckpt import orbax as ox


def _trainer():
    from sigma0_b200.models import preset_args
    from sigma0_b200.train.trainer import Trainer
    a = preset_args("smoke", d_model=32, mamba3_d_state=16, mamba3_headdim=16, n_messages=4, micro_bsz=2)
    return Trainer(a, device=torch.device("cpu"), total_steps=10, seed=0)


def test_orbax_roundtrip_is_bit_exact(tmp_path):
    tr = _trainer()
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    ds = LobWindowDataset.from_days(make_sequences(2, 5, seed=0), 4, token_mode="22tok")
    tr.train_step(collate([ds[0], ds[1]]))
    mgr = CheckpointManager(str(tmp_path), fmt="orbax")
    mgr.save(1, tr, metrics={"loss": 1.0}, config={"d_model": 32})
    d = tmp_path / "1"
    assert (d / "state" / "_METADATA").exists() and (d / "metadata" / "metadata").exists()
    assert (d / "_CHECKPOINT_METADATA").exists() and mgr.verify(1)
    keys = json.loads((d / "state" / "_METADATA").read_text())["tree_metadata"]
    assert "('params', 'decoder', 'kernel')" in keys or any(k.startswith("('params',") for k in keys)
    tr2 = _trainer()
    with torch.no_grad():
        for p in tr2.model.parameters():
            p.zero_()
    meta = CheckpointManager(str(tmp_path)).restore(tr2)
    assert meta["restored_step"] == 1
    for (n, a), (_, b) in zip(tr.model.named_parameters(), tr2.model.named_parameters()):
        assert torch.equal(a, b), n
    assert torch.equal(tr.opt.m, tr2.opt.m) and torch.equal(tr.opt.v, tr2.opt.v)
    assert tr2.opt.step_count == tr.opt.step_count


def _write_chunked(path, a, chunks, compressor="zlib", skip_zero_chunks=True, dtype=None):
    os.makedirs(path)
    hdr = {"zarr_format": 2, "shape": list(a.shape), "chunks": list(chunks), "dtype": dtype or "<f4",
           "compressor": {"id": compressor, "level": 3} if compressor else None, "fill_value": 0.0,
           "filters": None, "order": "C"}
    (open(os.path.join(path, ".zarray"), "w")).write(json.dumps(hdr))
    grid = [range(-(-s // c)) for s, c in zip(a.shape, chunks)]
    for idx in np.ndindex(*[len(g) for g in grid]):
        blk = np.zeros(chunks, dtype=a.dtype)
        sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, a.shape))
        part = a[sl]
        blk[tuple(slice(0, x.stop - x.start) for x in sl)] = part
        if skip_zero_chunks and a.ndim and not part.any():
            continue
        raw = blk.tobytes()
        with open(os.path.join(path, ".".join(map(str, idx)) if idx else "0"), "wb") as f:
            f.write(zlib.compress(raw) if compressor == "zlib" else raw)


def test_reference_layout_restores_into_lob_model(tmp_path):
    tr = _trainer()
    step = tmp_path / "7"
    state = step / "state"
    os.makedirs(state)
    rng = np.random.default_rng(0)
    md = {}
    want = {}
    for i, (n, p) in enumerate(tr.model.named_parameters()):
        from sigma0_b200.ckpt import flax_path
        kp = tuple(flax_path(n).split("/"))
        a = rng.standard_normal(tuple(p.shape)).astype(np.float32)
        if a.ndim >= 2:
            a[: a.shape[0] // 2] = 0                  # whole zero chunks are left out (fill value)
        want[kp] = a
        d = str(state / ".".join(kp))
        if i % 3 == 2 and a.ndim >= 1:                # bfloat16 storage for some leaves
            u16 = (a.view(np.uint32) >> 16).astype(np.uint16)
            want[kp] = ((u16.astype(np.uint32)) << 16).view(np.float32)
            _write_chunked(d, u16, tuple(max(1, s // 2) for s in a.shape), dtype="bfloat16")
        else:
            _write_chunked(d, a, tuple(max(1, s // 3) for s in a.shape) if a.ndim else ())
        md[str(kp)] = {"key_metadata": [], "value_metadata": {"value_type": "jax.Array", "skip_deserialize": False}}
    # the reference's train state also holds an optimizer state and a step
    _write_chunked(str(state / "step"), np.asarray(3, dtype=np.int32), (), compressor=None, dtype="<i4")
    md[str(("step",))] = {"key_metadata": [], "value_metadata": {}}
    (state / "_METADATA").write_text(json.dumps({"tree_metadata": md, "use_zarr3": False}))
    os.makedirs(step / "metadata")
    (step / "metadata" / "metadata").write_text(json.dumps({"config": {"d_model": 32}}))
    (step / "_CHECKPOINT_METADATA").write_text("{}")
    mgr = CheckpointManager(str(tmp_path))
    assert mgr.steps() == [7] and mgr.verify(7)
    mgr.restore(tr, params_only=True)
    from sigma0_b200.ckpt import flax_path
    for n, p in tr.model.named_parameters():
        assert np.array_equal(p.detach().numpy(), want[tuple(flax_path(n).split("/"))]), n


def test_ocdbt_and_unknown_codecs_are_refused(tmp_path):
    d = tmp_path / "state"
    os.makedirs(d)
    (d / "manifest.ocdbt").write_bytes(b"\0")
    with pytest.raises(OrbaxFormatError, match="OCDBT"):
        read_standard_item(str(d))
    z = tmp_path / "z"
    _write_chunked(str(z), np.ones((4,), np.float32), (4,), compressor=None)
    hdr = json.loads((z / ".zarray").read_text())
    hdr["compressor"] = {"id": "blosc", "cname": "lz4", "clevel": 5}
    (z / ".zarray").write_text(json.dumps(hdr))
    with pytest.raises(OrbaxFormatError, match="blosc"):
        ox.read_zarr(str(z))
