"""Orbax ``StandardSave`` / ``JsonSave`` checkpoint layout, read and written without Orbax,
TensorStore or JAX (none is installed here).

The reference saves ``ocp.args.Composite(state=StandardSave(train_state),
metadata=JsonSave(...))`` through an Orbax ``CheckpointManager``
(``src/base_model/training/state.py:91-110``) and, when Orbax's own restore fails, reads
the parameter arrays back with TensorStore from the ``state`` item's ``_METADATA`` tree
(``:190-262``).  One step directory looks like::

    <base>/<step>/_CHECKPOINT_METADATA         JSON: item handlers, timestamps
    <base>/<step>/metadata/metadata            JSON item (config, metrics, ...)
    <base>/<step>/state/_METADATA              JSON: {"tree_metadata": {"('params', 'a', 'b')": {...}},
                                                      "use_zarr3": false}
    <base>/<step>/state/params.a.b/.zarray     zarr v2 array header
    <base>/<step>/state/params.a.b/0.0         chunk files ("." separated chunk keys)

This module writes that layout with one chunk per array (zarr v2, C order, no compressor or
zlib) and reads zarr v2 arrays with several chunks, missing chunks (fill value) and the
``null`` / ``zlib`` / ``gzip`` / ``zstd`` compressors, and zarr v3 arrays (``zarr.json``:
regular chunk grid, ``default`` or ``v2`` chunk keys, the ``transpose`` / ``bytes`` /
``zstd`` / ``gzip`` / ``crc32c`` codecs, ``sharding_indexed`` shards; zstd through the
system libzstd when the zstandard module is absent).  Arrays stored in an OCDBT database
(``manifest.ocdbt``) or with the ``blosc`` codec are refused with a clear error.
"""
from __future__ import annotations

import ast
import gzip
import json
import os
import time
import zlib
from typing import List, Any, Dict, Iterable, Optional, Tuple

import numpy as np

KeyPath = Tuple[str, ...]


class OrbaxFormatError(RuntimeError):
    pass


_DTYPES = {"<f4": np.float32, "<f8": np.float64, "<f2": np.float16, "<i4": np.int32, "<i8": np.int64,
           "|u1": np.uint8, "|i1": np.int8, "|b1": np.bool_, "<u4": np.uint32, "<u2": np.uint16, "<i2": np.int16}


def _dtype_str(a: np.ndarray) -> str:
    for k, v in _DTYPES.items():
        if a.dtype == np.dtype(v):
            return k
    raise OrbaxFormatError(f"dtype {a.dtype} has no zarr v2 code here")


def _parse_dtype(code) -> Tuple[np.dtype, bool]:
    """(numpy storage dtype, is_bfloat16)."""
    if code == "bfloat16":                       # TensorStore's zarr v2 name for bfloat16
        return np.dtype(np.uint16), True
    if isinstance(code, str) and code in _DTYPES:
        return np.dtype(_DTYPES[code]), False
    if isinstance(code, str) and code[0] in "<>|=":
        return np.dtype(code), False
    raise OrbaxFormatError(f"unsupported zarr dtype {code!r}")


def _bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------------------
# one zarr v2 array
# ---------------------------------------------------------------------------------------------
def write_zarr(path: str, a: np.ndarray, compress: bool = False) -> None:
    os.makedirs(path, exist_ok=True)
    a = np.ascontiguousarray(a)
    hdr = {"zarr_format": 2, "shape": list(a.shape), "chunks": list(a.shape) or [],
           "dtype": _dtype_str(a), "compressor": {"id": "zlib", "level": 1} if compress else None,
           "fill_value": None, "filters": None, "order": "C", "dimension_separator": "."}
    with open(os.path.join(path, ".zarray"), "w") as f:
        json.dump(hdr, f)
    raw = a.tobytes()
    key = ".".join("0" for _ in a.shape) if a.ndim else "0"
    with open(os.path.join(path, key), "wb") as f:
        f.write(zlib.compress(raw, 1) if compress else raw)


def _decode(buf: bytes, comp: Optional[dict]) -> bytes:
    if comp is None:
        return buf
    cid = comp.get("id")
    if cid == "zlib":
        return zlib.decompress(buf)
    if cid == "gzip":
        return gzip.decompress(buf)
    if cid == "zstd":
        return _zstd_decompress(buf)
    raise OrbaxFormatError(f"compressor {cid!r} is not available in this image (only zlib / gzip / zstd / none)")


def _zstd_decompress(buf: bytes) -> bytes:
    try:
        import zstandard
        return zstandard.ZstdDecompressor().decompressobj().decompress(buf)
    except ImportError:
        from ..utils import zstd
        return zstd.decompress(buf)


def read_zarr(path: str) -> np.ndarray:
    with open(os.path.join(path, ".zarray")) as f:
        hdr = json.load(f)
    if hdr.get("zarr_format") != 2:
        raise OrbaxFormatError(f"{path}: only zarr v2 arrays are read")
    if hdr.get("filters"):
        raise OrbaxFormatError(f"{path}: zarr filters are not supported")
    dt, bf16 = _parse_dtype(hdr["dtype"])
    shape, chunks = tuple(hdr["shape"]), tuple(hdr["chunks"])
    order = hdr.get("order", "C")
    sep = hdr.get("dimension_separator", ".")
    fill = hdr.get("fill_value")
    out = np.full(shape, 0 if fill in (None, "NaN") else fill, dtype=dt)
    if fill == "NaN":
        out[...] = np.nan
    if not shape:
        keys = [((), "0")]
    else:
        grid = [range(-(-s // c)) for s, c in zip(shape, chunks)]
        keys = [(idx, sep.join(map(str, idx))) for idx in np.ndindex(*[len(g) for g in grid])]
    for idx, key in keys:
        fp = os.path.join(path, key)
        if not os.path.exists(fp):
            continue                                  # an all-fill-value chunk is not stored
        with open(fp, "rb") as f:
            raw = _decode(f.read(), hdr.get("compressor"))
        blk = np.frombuffer(raw, dtype=dt).reshape(chunks if shape else (), order=order)
        if shape:
            sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, shape))
            out[sl] = blk[tuple(slice(0, x.stop - x.start) for x in sl)]
        else:
            out[...] = blk
    return _bf16_to_f32(out) if bf16 else out


_V3_TYPES = {"bfloat16": "bfloat16", "float32": "<f4", "float64": "<f8", "float16": "<f2", "int8": "|i1",
             "int16": "<i2", "int32": "<i4", "int64": "<i8", "uint8": "|u1", "uint16": "<u2", "uint32": "<u4",
             "uint64": "<u8", "bool": "|b1"}


def _decode_v3(raw: bytes, codecs: List[dict], shape: Tuple[int, ...], dt: np.dtype, path: str) -> np.ndarray:
    """One chunk through a zarr v3 codec chain (decoded in reverse order)."""
    transpose, endian, byte_codecs = None, "little", []
    for c in codecs:
        name, conf = c["name"], c.get("configuration", {})
        if name == "transpose":
            transpose = tuple(conf["order"])
        elif name == "bytes":
            endian = conf.get("endian", "little")
        elif name in ("zstd", "gzip", "crc32c"):
            byte_codecs.append(name)
        else:
            raise OrbaxFormatError(f"{path}: zarr v3 codec {name!r} is not supported here")
    for name in reversed(byte_codecs):
        if name == "zstd":
            raw = _zstd_decompress(raw)
        elif name == "gzip":
            raw = gzip.decompress(raw)
        else:
            raw = raw[:-4]                            # the trailing crc32c (not verified here)
    sdt = dt.newbyteorder(">" if endian == "big" else "<") if dt.itemsize > 1 else dt
    inner = tuple(shape[i] for i in transpose) if transpose else shape
    blk = np.frombuffer(raw, dtype=sdt).astype(dt).reshape(inner)
    return np.transpose(blk, np.argsort(transpose)) if transpose else blk


def _place(out: np.ndarray, blk: np.ndarray, idx, chunks) -> None:
    if not out.shape:
        out[...] = blk
        return
    sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, out.shape))
    if any(x.start >= x.stop for x in sl):
        return
    out[sl] = blk[tuple(slice(0, x.stop - x.start) for x in sl)]


def _shard_chunks(raw: bytes, conf: dict, shard_shape, dt, path: str):
    """(inner chunk index, decoded inner chunk) of one ``sharding_indexed`` shard: the index is
    a (n_inner, 2) uint64 array of (offset, nbytes) -- all ones marks an empty chunk -- encoded
    with ``index_codecs`` at the start or the end of the shard."""
    inner = tuple(conf["chunk_shape"])
    grid = [s // c for s, c in zip(shard_shape, inner)]
    n = int(np.prod(grid)) if grid else 1
    icodecs = conf.get("index_codecs", [{"name": "bytes", "configuration": {"endian": "little"}},
                                        {"name": "crc32c"}])
    isize = 16 * n + (4 if any(c["name"] == "crc32c" for c in icodecs) else 0)
    at_start = conf.get("index_location", "end") == "start"
    ibytes = raw[:isize] if at_start else raw[-isize:]
    index = _decode_v3(ibytes, icodecs, tuple(grid) + (2,), np.dtype("<u8"), path)
    for j, idx in enumerate(np.ndindex(*grid)):
        off, nb = int(index[idx][0]), int(index[idx][1])
        if off == 2 ** 64 - 1 and nb == 2 ** 64 - 1:
            continue
        yield idx, _decode_v3(raw[off:off + nb], conf["codecs"], inner, dt, path)


def read_zarr3(path: str) -> np.ndarray:
    """A zarr v3 array (``zarr.json``) with a regular chunk grid, plain or ``sharding_indexed``
    chunks."""
    with open(os.path.join(path, "zarr.json")) as f:
        hdr = json.load(f)
    if hdr.get("zarr_format") != 3 or hdr.get("node_type", "array") != "array":
        raise OrbaxFormatError(f"{path}: not a zarr v3 array")
    grid = hdr["chunk_grid"]
    if grid.get("name") != "regular":
        raise OrbaxFormatError(f"{path}: chunk grid {grid.get('name')!r} is not read here")
    chunks = tuple(grid["configuration"]["chunk_shape"])
    shape = tuple(hdr["shape"])
    dt, bf16 = _parse_dtype(_V3_TYPES.get(hdr["data_type"], hdr["data_type"]))
    enc = hdr.get("chunk_key_encoding", {"name": "default"})
    sep = enc.get("configuration", {}).get("separator", "/" if enc.get("name", "default") == "default" else ".")
    codecs = hdr.get("codecs", [])
    shard = codecs[0] if len(codecs) == 1 and codecs[0]["name"] == "sharding_indexed" else None
    fill = hdr.get("fill_value", 0)
    out = np.full(shape, 0 if fill in (None, "NaN") else fill, dtype=dt)
    if fill == "NaN":
        out[...] = np.nan
    n_grid = [-(-s // c) for s, c in zip(shape, chunks)] if shape else []
    for idx in (np.ndindex(*n_grid) if shape else [()]):
        if enc.get("name", "default") == "default":
            key = sep.join(["c"] + [str(i) for i in idx])
        else:
            key = sep.join(str(i) for i in idx) if idx else "0"
        fp = os.path.join(path, *key.split("/"))
        if not os.path.exists(fp):
            continue
        with open(fp, "rb") as f:
            raw = f.read()
        if shard is None:
            _place(out, _decode_v3(raw, codecs, chunks if shape else (), dt, path), idx, chunks)
            continue
        conf = shard["configuration"]
        inner = tuple(conf["chunk_shape"])
        for j, blk in _shard_chunks(raw, conf, chunks, dt, path):
            # inner chunk j of shard idx covers the global chunk idx * (shard / inner) + j
            gidx = tuple(i * (c // k) + jj for i, c, k, jj in zip(idx, chunks, inner, j))
            _place(out, blk, gidx, inner)
    return _bf16_to_f32(out) if bf16 else out


# ---------------------------------------------------------------------------------------------
# a StandardSave item (a pytree of arrays) and a whole step
# ---------------------------------------------------------------------------------------------
def _keystr(kp: KeyPath) -> str:
    return str(tuple(kp))


def write_standard_item(item_dir: str, tree: Dict[KeyPath, np.ndarray], compress: bool = False) -> None:
    os.makedirs(item_dir, exist_ok=True)
    md = {}
    for kp, a in tree.items():
        write_zarr(os.path.join(item_dir, ".".join(kp)), np.asarray(a), compress)
        md[_keystr(kp)] = {"key_metadata": [{"key": k, "key_type": 2} for k in kp],
                           "value_metadata": {"value_type": "np.ndarray", "skip_deserialize": False}}
    with open(os.path.join(item_dir, "_METADATA"), "w") as f:
        json.dump({"tree_metadata": md, "use_zarr3": False}, f)


def read_standard_item(item_dir: str, prefix: Optional[str] = None) -> Dict[KeyPath, np.ndarray]:
    """Every array of the item (those under the top-level key ``prefix`` only, if given)."""
    if os.path.exists(os.path.join(item_dir, "manifest.ocdbt")) or \
            any(d.startswith("ocdbt.process") for d in os.listdir(item_dir)):
        raise OrbaxFormatError(f"{item_dir} is an OCDBT checkpoint; only the plain zarr layout "
                               "(use_ocdbt=False) is read here")
    mp = os.path.join(item_dir, "_METADATA")
    if os.path.exists(mp):
        with open(mp) as f:
            meta = json.load(f)
        kps = [tuple(ast.literal_eval(k)) for k in meta["tree_metadata"]]
    else:                                           # older layouts: one directory per array
        kps = [tuple(d.split(".")) for d in os.listdir(item_dir)
               if os.path.exists(os.path.join(item_dir, d, ".zarray"))]
    out = {}
    for kp in kps:
        if prefix is not None and kp[0] != prefix:
            continue
        d = os.path.join(item_dir, ".".join(kp))
        if os.path.exists(os.path.join(d, ".zarray")):
            out[kp] = read_zarr(d)
        elif os.path.exists(os.path.join(d, "zarr.json")):
            out[kp] = read_zarr3(d)
    return out


def write_step(step_dir: str, state: Dict[KeyPath, np.ndarray], metadata: Dict[str, Any],
               compress: bool = False) -> None:
    """One Orbax step directory: the ``state`` pytree and the ``metadata`` JSON item."""
    write_standard_item(os.path.join(step_dir, "state"), state, compress)
    os.makedirs(os.path.join(step_dir, "metadata"), exist_ok=True)
    with open(os.path.join(step_dir, "metadata", "metadata"), "w") as f:
        json.dump(metadata, f, indent=1)
    now = time.time_ns()
    with open(os.path.join(step_dir, "_CHECKPOINT_METADATA"), "w") as f:
        json.dump({"item_handlers": {"state": "orbax.checkpoint._src.handlers.standard_checkpoint_handler."
                                              "StandardCheckpointHandler",
                                     "metadata": "orbax.checkpoint._src.handlers.json_checkpoint_handler."
                                                 "JsonCheckpointHandler"},
                   "metrics": {}, "performance_metrics": {}, "init_timestamp_nsecs": now,
                   "commit_timestamp_nsecs": now, "custom_metadata": {}}, f)


def is_orbax_step(step_dir: str) -> bool:
    return os.path.exists(os.path.join(step_dir, "state", "_METADATA")) or \
        os.path.exists(os.path.join(step_dir, "_CHECKPOINT_METADATA"))


def params_tree(model) -> Dict[KeyPath, np.ndarray]:
    """A torch LOB model's parameters as Flax key paths ``('params', ...)`` -> float32 arrays."""
    from .checkpoint import flax_path
    return {tuple(flax_path(n).split("/")): p.detach().float().cpu().numpy() for n, p in model.named_parameters()}


def load_params_into(model, tree: Dict[KeyPath, np.ndarray], strict: bool = True) -> Iterable[str]:
    """Copy ``('params', ...)`` arrays into the model by Flax path; returns the paths missing
    from the tree (an error with ``strict``)."""
    import torch
    from .checkpoint import flax_path
    missing = []
    with torch.no_grad():
        for n, p in model.named_parameters():
            kp = tuple(flax_path(n).split("/"))
            a = tree.get(kp)
            if a is None:
                missing.append("/".join(kp))
                continue
            if tuple(a.shape) != tuple(p.shape):
                raise OrbaxFormatError(f"shape mismatch for {'/'.join(kp)}: {a.shape} vs {tuple(p.shape)}")
            p.copy_(torch.from_numpy(np.ascontiguousarray(a)).to(p.dtype))
    if strict and missing:
        raise OrbaxFormatError(f"checkpoint lacks {len(missing)} parameters, e.g. {missing[:3]}")
    return missing
