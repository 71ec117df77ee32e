"""Pack, verify and unpack run trees (inference outputs, checkpoints).

The reference packs inference trees into SquashFS images and overlays them
(``lobpipeline/storage/sqfs.py``, ``pipeline/package_run.py``); ``mksquashfs`` is
not part of this image, so a run is packed into a deterministic tar (sorted
members, zeroed owners and timestamps) with a SHA-256 manifest of every file;
``verify`` re-hashes an archive's members against the manifest and ``unpack``
restores it (refusing members that would escape the target directory).
"""
from __future__ import annotations

import hashlib
import io
import json
import os
import tarfile
from typing import Dict

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
