"""Checkpoint save / restore for the flat-buffer trainer.

Two formats under the reference's Orbax-manager directory layout and retention
(``run/base_model/runtime/train.py:538-578``): ``fmt="native"`` (default) writes raw
little-endian float32 flat buffers plus a JSON leaf table with SHA-256 hashes (fast,
sharded moments); ``fmt="orbax"`` writes the Orbax ``StandardSave`` / ``JsonSave`` layout
(zarr v2 arrays under Flax key paths, ``ckpt/orbax.py``).  ``restore`` reads either, by
Flax path; Orbax checkpoints stored in OCDBT databases are refused (no codec here).
``export_params_npz`` exchanges weights by Flax path.  Native files:

    <base>/<step>/state/params.f32          float32 flat parameter buffer
    <base>/<step>/state/adam_m.r<k>.f32     Adam first moment, rank k's shard
    <base>/<step>/state/adam_v.r<k>.f32     Adam second moment, rank k's shard
    <base>/<step>/state/index.json          leaf table: Flax path, shape, offset
    <base>/<step>/metadata/metadata         JSON: step, config, metrics, world, hashes

Parameters are addressed by their Flax paths (``params/message_encoder/...``),
so a parameters-only restore works across optimizer layouts and world sizes.
The flat buffers are written with one host copy per buffer (pinned staging,
then a background writer thread), so a save costs the step one device->host
copy.  Each step directory is written under a temporary name and renamed
into place, so a crash never leaves a half-written checkpoint that looks
complete; every file carries a SHA-256 in the metadata, checked on restore.

Retention follows Orbax ``max_to_keep`` / ``keep_period``: the newest
``max_to_keep`` steps are kept, plus every step divisible by ``keep_period``.
``restore`` falls back to the newest *intact* checkpoint when the latest one
fails verification.  ``remap_step`` implements the elastic step remap of
``train.py:296-325`` (same number of samples seen when the global batch
changes).
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import threading
from typing import Dict, List, Optional

import numpy as np
import torch


def flax_path(name: str) -> str:
    """Torch parameter name -> Flax parameter path.  The context-parallel wrappers hold the
    block they wrap as ``inner``; that segment is dropped so a wrapped model saves and loads
    under the same paths as the plain one."""
    return "params/" + "/".join(p for p in name.split(".") if p != "inner")


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 24), b""):
            h.update(blk)
    return h.hexdigest()


def remap_step(step: int, old_global_batch: int, new_global_batch: int) -> int:
    """Step index that has seen the same number of sequences under a new global batch."""
    if old_global_batch == new_global_batch or new_global_batch <= 0:
        return step
    return (step * old_global_batch) // new_global_batch


class CheckpointError(RuntimeError):
    pass


class CheckpointManager:
    def __init__(self, base_dir: str, max_to_keep: int = 10, keep_period: int = 5, rank: int = 0, world: int = 1,
                 barrier=None, fmt: str = "native"):
        if fmt not in ("native", "orbax"):
            raise ValueError(f"checkpoint format must be 'native' or 'orbax', not {fmt!r}")
        self.fmt = fmt
        self.base = base_dir
        self.max_to_keep, self.keep_period = max_to_keep, keep_period
        self.rank, self.world = rank, world
        self.barrier = barrier or (lambda: None)
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None
        os.makedirs(base_dir, exist_ok=True)

    # -- discovery ------------------------------------------------------------------------
    def steps(self) -> List[int]:
        out = []
        for d in os.listdir(self.base):
            if d.isdigit() and os.path.isfile(os.path.join(self.base, d, "metadata", "metadata")):
                out.append(int(d))
        return sorted(out)

    def latest_step(self) -> Optional[int]:
        s = self.steps()
        return s[-1] if s else None

    # -- save -------------------------------------------------------------------------------
    def wait(self):
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            e, self._error = self._error, None
            raise CheckpointError(f"asynchronous checkpoint write failed: {e}") from e

    def save(self, step: int, trainer, metrics: Optional[Dict] = None, config: Optional[Dict] = None,
             blocking: bool = False) -> str:
        """Snapshot ``trainer`` (flat params, Adam moments, step) as ``<base>/<step>``."""
        self.wait()
        if self.fmt == "orbax":
            return self._save_orbax(step, trainer, metrics, config)
        opt = trainer.opt
        tmp = os.path.join(self.base, f".{step}.tmp")
        final = os.path.join(self.base, str(step))
        if self.rank == 0:
            shutil.rmtree(tmp, ignore_errors=True)
            os.makedirs(os.path.join(tmp, "state"), exist_ok=True)
            os.makedirs(os.path.join(tmp, "metadata"), exist_ok=True)
        self.barrier()
        # device -> pinned host, ordered on the current stream
        m_local, v_local = opt.local_moments()
        pin = opt.device.type == "cuda"
        host = {}
        for key, t in (("adam_m", m_local), ("adam_v", v_local)) + ((("params", opt.flat),) if self.rank == 0 else ()):
            h = torch.empty(t.numel(), dtype=torch.float32, pin_memory=pin)
            h.copy_(t, non_blocking=pin)
            host[key] = h
        if pin:
            torch.cuda.current_stream().synchronize()
        index = {"leaves": [{"name": n, "path": flax_path(n), "shape": list(p.shape), "offset": opt.slices[n][0]}
                            for n, p in zip(opt.names, opt.params_in_order())],
                 "numel": opt.numel, "n_ssm": opt.n_ssm, "shard_bounds": opt.shard_bounds(), "world": self.world}
        meta = {"step": int(step), "optimizer_step": int(opt.step_count), "trainer_step": int(trainer.step_idx),
                "global_batch": int(getattr(trainer, "global_batch", 0)), "world": self.world,
                "config": config or {}, "metrics": metrics or {}}
        rank = self.rank
        # FSDP-sharded kernels (parallel/fsdp.py): every rank takes part in gathering the full
        # fp32 kernels, rank 0 writes them by Flax path; each rank writes its moment shards
        fsdp = getattr(trainer, "fsdp", None)
        fsdp_host = None
        if fsdp is not None:
            names = {id(p): n for n, p in trainer.model.named_parameters()}
            full = fsdp.full_parameters()
            fsdp_host = {"params": {flax_path(names[id(p)]): t.cpu().numpy() for p, t in full.items()}
                         if self.rank == 0 else None,
                         "m": torch.cat([u.m for u in fsdp.units]).cpu().numpy(),
                         "v": torch.cat([u.v for u in fsdp.units]).cpu().numpy()}
            meta["fsdp_step"] = int(fsdp.step_count)

        def write():
            try:
                st = os.path.join(tmp, "state")
                files = {}
                for key, h in host.items():
                    name = "params.f32" if key == "params" else f"{key}.r{rank}.f32"
                    p = os.path.join(st, name)
                    h.numpy().tofile(p)
                    files[name] = _sha256(p)
                if fsdp_host is not None:
                    for key in ("m", "v"):
                        name = f"fsdp_{key}.r{rank}.f32"
                        fsdp_host[key].tofile(os.path.join(st, name))
                        files[name] = _sha256(os.path.join(st, name))
                    if fsdp_host["params"] is not None:
                        name = "fsdp_params.npz"
                        np.savez(os.path.join(st, name), **fsdp_host["params"])
                        files[name] = _sha256(os.path.join(st, name))
                with open(os.path.join(st, f"hashes.r{rank}.json"), "w") as f:
                    json.dump(files, f)
                if rank == 0:
                    with open(os.path.join(st, "index.json"), "w") as f:
                        json.dump(index, f)
            except BaseException as e:  # surfaced by wait()
                self._error = e

        if blocking or self.world > 1:
            write()
            if self._error is not None:
                self.wait()
            self._finish(tmp, final, meta)
        else:
            def job():
                write()
                if self._error is None:
                    try:
                        self._finish(tmp, final, meta)
                    except BaseException as e:
                        self._error = e
            self._thread = threading.Thread(target=job, daemon=True)
            self._thread.start()
        return final

    def _finish(self, tmp: str, final: str, meta: Dict):
        self.barrier()
        if self.rank == 0:
            st = os.path.join(tmp, "state")
            hashes = {}
            for f in sorted(os.listdir(st)):
                if f.startswith("hashes.r"):
                    with open(os.path.join(st, f)) as fh:
                        hashes.update(json.load(fh))
            hashes["index.json"] = _sha256(os.path.join(st, "index.json"))
            meta["sha256"] = hashes
            with open(os.path.join(tmp, "metadata", "metadata"), "w") as f:
                json.dump(meta, f, indent=1)
            shutil.rmtree(final, ignore_errors=True)
            os.replace(tmp, final)
            self._retain()
        self.barrier()

    def _retain(self):
        steps = self.steps()
        keep = set(steps[-self.max_to_keep:]) if self.max_to_keep > 0 else set(steps)
        for s in steps:
            if s not in keep and not (self.keep_period and s % self.keep_period == 0):
                shutil.rmtree(os.path.join(self.base, str(s)), ignore_errors=True)

    def _save_orbax(self, step: int, trainer, metrics, config) -> str:
        """The step in the Orbax layout (``ckpt/orbax.py``): ``state`` = {params, step,
        opt_state/{mu, nu} (unsharded optimizers)}, ``metadata`` = the JSON record."""
        from . import orbax as ox
        if getattr(trainer, "fsdp", None) is not None:
            raise CheckpointError("the Orbax layout is written for replicated parameters; save FSDP runs with "
                                  "fmt='native'")
        opt = trainer.opt
        tmp = os.path.join(self.base, f".{step}.tmp")
        final = os.path.join(self.base, str(step))
        if self.rank == 0:
            tree = ox.params_tree(trainer.model)
            tree[("step",)] = np.asarray(opt.step_count, dtype=np.int64)
            if not getattr(opt, "sharded", False):
                for n, p in zip(opt.names, opt.params_in_order()):
                    a, b = opt.slices[n]
                    kp = tuple(flax_path(n).split("/"))[1:]
                    tree[("opt_state", "mu") + kp] = opt.m[a:b].view(p.shape).detach().cpu().numpy()
                    tree[("opt_state", "nu") + kp] = opt.v[a:b].view(p.shape).detach().cpu().numpy()
            meta = {"step": int(step), "optimizer_step": int(opt.step_count), "trainer_step": int(trainer.step_idx),
                    "global_batch": int(getattr(trainer, "global_batch", 0)), "world": self.world,
                    "config": config or {}, "metrics": metrics or {}, "format": "orbax"}
            shutil.rmtree(tmp, ignore_errors=True)
            ox.write_step(tmp, tree, meta)
            shutil.rmtree(final, ignore_errors=True)
            os.replace(tmp, final)
            self._retain()
        self.barrier()
        return final

    # -- restore ----------------------------------------------------------------------------
    def verify(self, step: int) -> bool:
        d = os.path.join(self.base, str(step))
        from . import orbax as ox
        if ox.is_orbax_step(d):      # no hashes in that layout: every listed array must have its header
            try:
                with open(os.path.join(d, "state", "_METADATA")) as f:
                    import ast
                    kps = [ast.literal_eval(k) for k in json.load(f)["tree_metadata"]]
                return all(any(os.path.exists(os.path.join(d, "state", ".".join(kp), h)) for h in (".zarray", "zarr.json"))
                           for kp in kps)
            except (OSError, KeyError, ValueError, SyntaxError):
                return False
        try:
            with open(os.path.join(d, "metadata", "metadata")) as f:
                meta = json.load(f)
            for name, h in meta["sha256"].items():
                if _sha256(os.path.join(d, "state", name)) != h:
                    return False
            return True
        except (OSError, KeyError, ValueError):
            return False

    def restore(self, trainer, step: Optional[int] = None, params_only: bool = False) -> Dict:
        """Load a checkpoint into ``trainer``; returns its metadata.

        ``step=None`` takes the newest checkpoint that verifies.  With
        ``params_only`` (the reference's ``--partial_restore`` fallback) only the
        parameters are read, by Flax path, so the optimizer layout may differ."""
        cands = [step] if step is not None else list(reversed(self.steps()))
        chosen = None
        for s in cands:
            if self.verify(s):
                chosen = s
                break
        if chosen is None:
            raise CheckpointError(f"no intact checkpoint in {self.base} (candidates {cands})")
        d = os.path.join(self.base, str(chosen))
        with open(os.path.join(d, "metadata", "metadata")) as f:
            meta = json.load(f)
        from . import orbax as ox
        if ox.is_orbax_step(d):
            return self._restore_orbax(trainer, d, meta, chosen, params_only)
        with open(os.path.join(d, "state", "index.json")) as f:
            index = json.load(f)
        opt = trainer.opt
        flat = np.fromfile(os.path.join(d, "state", "params.f32"), dtype=np.float32)
        by_path = {l["path"]: l for l in index["leaves"]}
        same_layout = (index["numel"] == opt.numel and
                       all(by_path.get(flax_path(n), {}).get("offset") == opt.slices[n][0] for n in opt.names))
        with torch.no_grad():
            if same_layout:
                opt.flat.copy_(torch.from_numpy(flat))
            else:
                for n, p in zip(opt.names, opt.params_in_order()):
                    leaf = by_path.get(flax_path(n))
                    if leaf is None:
                        raise CheckpointError(f"checkpoint has no leaf {flax_path(n)}")
                    if list(leaf["shape"]) != list(p.shape):
                        raise CheckpointError(f"shape mismatch for {flax_path(n)}: {leaf['shape']} vs {list(p.shape)}")
                    o = leaf["offset"]
                    p.copy_(torch.from_numpy(flat[o:o + p.numel()]).view_as(p))
            opt.refresh_shadow()
            if not params_only:
                if not same_layout:
                    raise CheckpointError("optimizer state needs the same parameter layout; use params_only=True")
                full = {}
                for key in ("adam_m", "adam_v"):
                    parts = [np.fromfile(os.path.join(d, "state", f"{key}.r{k}.f32"), dtype=np.float32)
                             for k in range(index["world"])]
                    full[key] = np.concatenate(parts) if index.get("shard_bounds") else parts[0]
                opt.load_full_moments(torch.from_numpy(full["adam_m"]), torch.from_numpy(full["adam_v"]),
                                      int(meta["optimizer_step"]))
                gb_new = int(getattr(trainer, "global_batch", 0))
                trainer.step_idx = remap_step(int(meta["trainer_step"]), int(meta.get("global_batch", 0)), gb_new)
        self._restore_fsdp(trainer, d, index, params_only)
        if getattr(trainer, "fsdp", None) is not None and not params_only:
            trainer.fsdp.step_count = int(meta.get("fsdp_step", 0))
        meta["restored_step"] = chosen
        return meta

    def _restore_fsdp(self, trainer, d: str, index: Dict, params_only: bool) -> None:
        """The FSDP-sharded kernels: full parameters by Flax path, re-sharded for this run; the
        moment shards when the world size is the same."""
        fsdp = getattr(trainer, "fsdp", None)
        path = os.path.join(d, "state", "fsdp_params.npz")
        if fsdp is None:
            return
        if not os.path.exists(path):
            raise CheckpointError(f"{d} has no FSDP kernels (saved without FSDP?)")
        arrs = np.load(path)
        names = {id(p): n for n, p in trainer.model.named_parameters()}
        full = {p: torch.from_numpy(arrs[flax_path(names[id(p)])]).to(fsdp.device)
                for p in fsdp.sharded_parameters()}
        fsdp.load_full_parameters(full)
        mp = os.path.join(d, "state", f"fsdp_m.r{self.rank}.f32")
        if not params_only and index.get("world") == self.world and os.path.exists(mp):
            m = torch.from_numpy(np.fromfile(mp, dtype=np.float32)).to(fsdp.device)
            v = torch.from_numpy(np.fromfile(os.path.join(d, "state", f"fsdp_v.r{self.rank}.f32"),
                                             dtype=np.float32)).to(fsdp.device)
            o = 0
            for u in fsdp.units:
                u.m.copy_(m[o:o + u.shard])
                u.v.copy_(v[o:o + u.shard])
                o += u.shard

    def _restore_orbax(self, trainer, d: str, meta: Dict, chosen: int, params_only: bool) -> Dict:
        from . import orbax as ox
        tree = ox.read_standard_item(os.path.join(d, "state"))
        opt = trainer.opt
        ox.load_params_into(trainer.model, {k: v for k, v in tree.items() if k[0] == "params"})
        with torch.no_grad():
            opt.refresh_shadow()
            has_mom = any(k[:2] == ("opt_state", "mu") for k in tree)
            if not params_only and has_mom:
                m = torch.zeros(opt.numel, dtype=torch.float32)
                v = torch.zeros(opt.numel, dtype=torch.float32)
                for n in opt.names:
                    a, b = opt.slices[n]
                    kp = tuple(flax_path(n).split("/"))[1:]
                    m[a:b] = torch.from_numpy(np.ascontiguousarray(tree[("opt_state", "mu") + kp])).reshape(-1)
                    v[a:b] = torch.from_numpy(np.ascontiguousarray(tree[("opt_state", "nu") + kp])).reshape(-1)
                opt.load_full_moments(m.to(opt.device), v.to(opt.device), int(meta.get("optimizer_step", 0)))
            if not params_only:
                trainer.step_idx = remap_step(int(meta.get("trainer_step", chosen)), int(meta.get("global_batch", 0)),
                                              int(getattr(trainer, "global_batch", 0)))
        meta["restored_step"] = chosen
        return meta

    def export_params_npz(self, trainer, path: str) -> None:
        """Parameters as one ``.npz`` keyed by Flax path (a framework-neutral export)."""
        opt = trainer.opt
        arrs = {flax_path(n): p.detach().float().cpu().numpy() for n, p in zip(opt.names, opt.params_in_order())}
        np.savez(path, **arrs)
