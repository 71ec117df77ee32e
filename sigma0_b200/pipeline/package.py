"""Pack, verify and unpack run trees (inference outputs, checkpoints).

The reference packs inference trees into SquashFS images and overlays them
(``lobpipeline/storage/sqfs.py``, ``pipeline/package_run.py``); ``mksquashfs`` is
not part of this image, so a run is packed into a deterministic tar (sorted
members, zeroed owners and timestamps) with a SHA-256 manifest of every file;
``verify`` re-hashes an archive's members against the manifest and ``unpack``
restores it (refusing members that would escape the target directory).  A packed tree
``<dir>.tar`` can be patched without repacking through ``<dir>.overlay`` (file overrides and
whiteouts), read through ``resolve`` as a merged directory, and read member by member with
``cat`` / ``listing``.

``package_run`` binds a finished benchmark run into one archive with the layout of the
reference's run package (``lobpipeline/pipeline/package_run.py``): ``manifest.json`` (run
name, the metric names of the scores, the file inventory), ``scores.json`` and the
predictions under ``predictions/`` copied verbatim, plus a sidecar ``index_<run>.json`` next
to the archive so consumers can list its contents without opening it.  ``plan_package``
validates the inputs and computes the paths without touching anything.
"""
from __future__ import annotations

import hashlib
import io
import json
import os
import shutil
import tarfile
import tempfile
from typing import Dict, List

MANIFEST = "MANIFEST.sha256.json"


def pack(root: str, archive: str) -> Dict[str, str]:
    files = []
    for d, dirs, fs in os.walk(root):
        dirs.sort()
        for f in sorted(fs):
            files.append(os.path.join(d, f))
    manifest = {}
    with tarfile.open(archive, "w") as tar:
        for p in sorted(files):
            rel = os.path.relpath(p, root).replace(os.sep, "/")
            data = open(p, "rb").read()
            manifest[rel] = hashlib.sha256(data).hexdigest()
            ti = tarfile.TarInfo(rel)
            ti.size, ti.mtime, ti.uid, ti.gid, ti.mode = len(data), 0, 0, 0, 0o644
            tar.addfile(ti, io.BytesIO(data))
        blob = json.dumps(manifest, indent=1, sort_keys=True).encode()
        ti = tarfile.TarInfo(MANIFEST)
        ti.size, ti.mtime, ti.mode = len(blob), 0, 0o644
        tar.addfile(ti, io.BytesIO(blob))
    return manifest


def verify(archive: str) -> Dict[str, list]:
    bad = {"mismatch": [], "missing": [], "extra": []}
    with tarfile.open(archive) as tar:
        manifest = json.load(tar.extractfile(MANIFEST))
        seen = set()
        for m in tar.getmembers():
            if m.name == MANIFEST:
                continue
            seen.add(m.name)
            h = hashlib.sha256(tar.extractfile(m).read()).hexdigest()
            if m.name not in manifest:
                bad["extra"].append(m.name)
            elif manifest[m.name] != h:
                bad["mismatch"].append(m.name)
        bad["missing"] = sorted(set(manifest) - seen)
    return bad


def unpack(archive: str, dest: str) -> None:
    dest = os.path.abspath(dest)
    with tarfile.open(archive) as tar:
        for m in tar.getmembers():
            target = os.path.abspath(os.path.join(dest, m.name))
            if not target.startswith(dest + os.sep):
                raise ValueError(f"archive member escapes the target: {m.name}")
        tar.extractall(dest)


IMAGE_SUFFIX = ".tar"
WHITEOUT = ".wh."


def image_for(directory: str) -> str:
    """The archive that stands for ``directory``: ``<directory>.tar``."""
    return os.path.normpath(directory) + IMAGE_SUFFIX


def overlay_for(directory: str) -> str:
    """The overlay directory of ``directory``'s archive: ``<directory>.overlay``."""
    return os.path.normpath(directory) + ".overlay"


def overlay_override(directory: str, relative: str, data) -> str:
    """Replace one file of a packed tree without repacking it (the reference's
    ``storage/sqfs.py:699-716``): ``relative`` is written into the overlay, and the next
    ``resolve`` reads it from there."""
    target = os.path.join(overlay_for(directory), relative)
    os.makedirs(os.path.dirname(target), exist_ok=True)
    wh = os.path.join(os.path.dirname(target), WHITEOUT + os.path.basename(target))
    if os.path.exists(wh):
        os.remove(wh)
    with open(target, "wb") as f:
        f.write(data.encode() if isinstance(data, str) else data)
    return target


def overlay_exclude(directory: str, relative: str) -> str:
    """Hide one file of a packed tree without repacking it (``storage/sqfs.py:717-742``):
    a whiteout marker ``.wh.<name>`` in the overlay (the overlay-filesystem naming; no
    device node, so no privileges are needed); ``resolve`` leaves the file out."""
    d = os.path.join(overlay_for(directory), os.path.dirname(relative))
    os.makedirs(d, exist_ok=True)
    shadow = os.path.join(d, os.path.basename(relative))
    if os.path.exists(shadow):
        os.remove(shadow)
    target = os.path.join(d, WHITEOUT + os.path.basename(relative))
    open(target, "wb").close()
    return target


def _apply_overlay(overlay: str, root: str) -> None:
    for d, _, fs in os.walk(overlay):
        rel = os.path.relpath(d, overlay)
        for f in fs:
            dst_dir = os.path.normpath(os.path.join(root, rel))
            if f.startswith(WHITEOUT):
                victim = os.path.join(dst_dir, f[len(WHITEOUT):])
                if os.path.isdir(victim):
                    shutil.rmtree(victim)
                elif os.path.exists(victim):
                    os.remove(victim)
            else:
                os.makedirs(dst_dir, exist_ok=True)
                shutil.copyfile(os.path.join(d, f), os.path.join(dst_dir, f))


class resolve:
    """``with resolve(path) as real_dir:`` a real directory for ``path`` (the reference's
    ``storage/sqfs.py:645-697``): ``path`` itself when it is a directory; else its archive
    (``<path>.tar``, or ``path`` when that is an archive) unpacked into a temporary
    directory with ``<path>.overlay`` applied on top (overrides replace files, whiteouts
    hide them), removed again on exit; ``require=False`` yields ``path`` unchanged when
    neither exists."""

    def __init__(self, path: str, tmp_root: str = None, require: bool = True):
        self.path, self.tmp_root, self.require, self.tmp = os.path.normpath(path), tmp_root, require, None

    def __enter__(self) -> str:
        if os.path.isdir(self.path):
            return self.path
        image = self.path if (self.path.endswith(IMAGE_SUFFIX) and os.path.isfile(self.path)) \
            else image_for(self.path)
        if not os.path.isfile(image):
            if self.require:
                raise FileNotFoundError(f"neither a directory nor a packed tree: {self.path}")
            return self.path
        self.tmp = tempfile.mkdtemp(prefix="resolve_", dir=self.tmp_root)
        unpack(image, self.tmp)
        man = os.path.join(self.tmp, MANIFEST)
        if os.path.exists(man):
            os.remove(man)
        base = self.path[:-len(IMAGE_SUFFIX)] if self.path.endswith(IMAGE_SUFFIX) else self.path
        if os.path.isdir(overlay_for(base)):
            _apply_overlay(overlay_for(base), self.tmp)
        return self.tmp

    def __exit__(self, *exc):
        if self.tmp:
            shutil.rmtree(self.tmp, ignore_errors=True)
        return False


def cat(archive: str, relative: str) -> bytes:
    """One member's bytes, without unpacking the archive."""
    with tarfile.open(archive) as tar:
        f = tar.extractfile(relative)
        if f is None:
            raise KeyError(f"{relative} is not a file in {archive}")
        return f.read()


def listing(archive: str) -> List[str]:
    """The relative paths of the packed files (the manifest left out)."""
    with tarfile.open(archive) as tar:
        return sorted(m.name for m in tar.getmembers() if m.isfile() and m.name != MANIFEST)


def plan_package(run_name: str, predictions_root: str, scores_path: str, output_dir: str) -> Dict[str, str]:
    """The package's paths after checking the inputs (no side effects)."""
    if not run_name or os.sep in run_name:
        raise ValueError(f"run_name must be a plain non-empty name, got {run_name!r}")
    if not os.path.isdir(predictions_root):
        raise FileNotFoundError(f"predictions directory not found: {predictions_root}")
    if not os.path.isfile(scores_path):
        raise FileNotFoundError(f"scores file not found: {scores_path}")
    return {"run_name": run_name, "predictions_root": os.path.abspath(predictions_root),
            "scores_path": os.path.abspath(scores_path),
            "archive": os.path.join(output_dir, f"{run_name}.tar"),
            "index": os.path.join(output_dir, f"index_{run_name}.json")}


def _metric_names(scores) -> List[str]:
    if isinstance(scores, dict):
        inner = scores.get("scores", scores)
        if isinstance(inner, dict):
            return sorted(str(k) for k in inner)
    return []


def package_run(run_name: str, predictions_root: str, scores_path: str, output_dir: str) -> Dict:
    """Stage ``manifest.json``, ``scores.json`` and ``predictions/`` and pack them into
    ``<output_dir>/<run_name>.tar`` (``pack``: deterministic, SHA-256 manifest); write the
    sidecar index.  Returns the index."""
    plan = plan_package(run_name, predictions_root, scores_path, output_dir)
    os.makedirs(output_dir, exist_ok=True)
    with open(plan["scores_path"]) as f:
        scores = json.load(f)
    with tempfile.TemporaryDirectory() as stage:
        shutil.copytree(plan["predictions_root"], os.path.join(stage, "predictions"))
        shutil.copyfile(plan["scores_path"], os.path.join(stage, "scores.json"))
        files = []
        for d, dirs, fs in os.walk(os.path.join(stage, "predictions")):
            dirs.sort()
            files += sorted(os.path.relpath(os.path.join(d, f), stage).replace(os.sep, "/") for f in fs)
        manifest = {"run_name": run_name, "metric_names": _metric_names(scores), "n_files": len(files),
                    "files": files}
        with open(os.path.join(stage, "manifest.json"), "w") as f:
            json.dump(manifest, f, indent=1, sort_keys=True)
        hashes = pack(stage, plan["archive"])
    index = {"run_name": run_name, "archive": os.path.basename(plan["archive"]),
             "metric_names": manifest["metric_names"], "members": sorted(hashes), "sha256": hashes}
    with open(plan["index"], "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)
    return index
