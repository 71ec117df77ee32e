"""zstd through the system libzstd (no zstandard module needed): ``.npy.zst`` day files and
zstd-compressed zarr chunks; zarr v3 arrays of an Orbax item read by the spec."""
import json
import os

import numpy as np
import pytest

from sigma0_b200.utils import zstd as Z

pytestmark = pytest.mark.skipif(not Z.available(), reason="no libzstd")


def test_roundtrip_and_concatenated_frames():
    d = os.urandom(3000) + b"x" * 70000
    c = Z.compress(d)
    assert len(c) < len(d) and Z.decompress(c) == d
    assert Z.decompress(c + Z.compress(b"tail")) == d + b"tail"
    with pytest.raises(Z.ZstdError):
        Z.decompress(b"not zstd at all")


def test_npy_zst_day_files(tmp_path):
    import io
    from sigma0_b200.data.lobster import resolve_day_files
    from sigma0_b200.data.masks import load_npy
    a = np.arange(60, dtype=np.int64).reshape(6, 10)
    for tag in ("message", "book"):
        buf = io.BytesIO()
        np.save(buf, a)
        (tmp_path / f"GOOG_2022-01-03_{tag}.npy.zst").write_bytes(Z.compress(buf.getvalue()))
    files = resolve_day_files(str(tmp_path))
    assert len(files) == 1 and files[0][0].endswith(".npy.zst")
    assert np.array_equal(load_npy(files[0][0]), a)


def _write_zarr3(path, arr, chunks, codecs, bf16=False, transpose=None):
    os.makedirs(path)
    hdr = {"zarr_format": 3, "node_type": "array", "shape": list(arr.shape),
           "data_type": "bfloat16" if bf16 else str(arr.dtype),
           "chunk_grid": {"name": "regular", "configuration": {"chunk_shape": list(chunks)}},
           "chunk_key_encoding": {"name": "default", "configuration": {"separator": "/"}},
           "fill_value": 0, "codecs": ([{"name": "transpose", "configuration": {"order": list(transpose)}}]
                                       if transpose else []) + codecs}
    json.dump(hdr, open(os.path.join(path, "zarr.json"), "w"))
    store = arr
    if bf16:
        store = (arr.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    grid = [-(-s // c) for s, c in zip(arr.shape, chunks)]
    for idx in np.ndindex(*grid):
        blk = np.zeros(chunks, store.dtype)
        sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, arr.shape))
        blk[tuple(slice(0, x.stop - x.start) for x in sl)] = store[sl]
        if transpose:
            blk = np.transpose(blk, transpose)
        raw = np.ascontiguousarray(blk).tobytes()
        if any(c["name"] == "zstd" for c in codecs):
            raw = Z.compress(raw)
        if idx == (0, 1):
            continue                                   # a missing chunk reads as the fill value
        fp = os.path.join(path, "c", *map(str, idx))
        os.makedirs(os.path.dirname(fp), exist_ok=True)
        open(fp, "wb").write(raw)


def test_zarr3_and_zstd_arrays_of_an_orbax_item(tmp_path):
    from sigma0_b200.ckpt import orbax as O
    rng = np.random.default_rng(0)
    w = rng.standard_normal((5, 7)).astype(np.float32)
    b = rng.standard_normal((5, 7)).astype(np.float32)
    item = tmp_path / "state"
    codecs = [{"name": "bytes", "configuration": {"endian": "little"}}, {"name": "zstd", "configuration": {"level": 1}}]
    _write_zarr3(str(item / "params.w"), w, (2, 4), codecs)
    _write_zarr3(str(item / "params.b"), b, (3, 3), codecs, bf16=True, transpose=(1, 0))
    md = {str(k): {} for k in (("params", "w"), ("params", "b"))}
    json.dump({"tree_metadata": md, "use_zarr3": True}, open(item / "_METADATA", "w"))
    got = O.read_standard_item(str(item))
    want_w = w.copy()
    want_w[0:2, 4:7] = 0.0                           # chunk (0, 1) was not written
    assert np.array_equal(got[("params", "w")], want_w)
    bf = ((b.view(np.uint32) >> 16) << 16).view(np.float32)
    want_b = bf.copy()
    want_b[0:3, 3:6] = 0.0
    assert np.array_equal(got[("params", "b")], want_b)
    # a zarr v2 chunk compressed with zstd
    d2 = tmp_path / "v2"
    os.makedirs(d2)
    json.dump({"zarr_format": 2, "shape": [4], "chunks": [4], "dtype": "<f4", "compressor": {"id": "zstd", "level": 3},
               "fill_value": 0, "order": "C", "filters": None}, open(d2 / ".zarray", "w"))
    (d2 / "0").write_bytes(Z.compress(np.arange(4, dtype=np.float32).tobytes()))
    assert np.array_equal(O.read_zarr(str(d2)), np.arange(4, dtype=np.float32))


def test_zarr3_sharded_array(tmp_path):
    """``sharding_indexed``: one shard file per (4, 4) block holding (2, 2) inner chunks, each
    zstd-compressed, with the (offset, nbytes) index (crc32c-suffixed) at the shard's end and
    one inner chunk left empty."""
    import struct
    import zlib
    from sigma0_b200.ckpt import orbax as O
    a = np.arange(6 * 8, dtype=np.float32).reshape(6, 8)
    path = tmp_path / "arr"
    os.makedirs(path)
    inner_codecs = [{"name": "bytes", "configuration": {"endian": "little"}}, {"name": "zstd", "configuration": {}}]
    idx_codecs = [{"name": "bytes", "configuration": {"endian": "little"}}, {"name": "crc32c"}]
    hdr = {"zarr_format": 3, "node_type": "array", "shape": [6, 8], "data_type": "float32",
           "chunk_grid": {"name": "regular", "configuration": {"chunk_shape": [4, 4]}},
           "chunk_key_encoding": {"name": "default"}, "fill_value": -1.0,
           "codecs": [{"name": "sharding_indexed", "configuration": {
               "chunk_shape": [2, 2], "codecs": inner_codecs, "index_codecs": idx_codecs,
               "index_location": "end"}}]}
    json.dump(hdr, open(path / "zarr.json", "w"))
    want = np.full((6, 8), -1.0, np.float32)
    for si in range(2):
        for sj in range(2):
            body, index = b"", []
            for ii in range(2):
                for jj in range(2):
                    r0, c0 = si * 4 + ii * 2, sj * 4 + jj * 2
                    if (si, sj, ii, jj) == (1, 1, 0, 1) or r0 >= 6:
                        index += [2 ** 64 - 1, 2 ** 64 - 1]          # empty inner chunk
                        continue
                    blk = a[r0:r0 + 2, c0:c0 + 2]
                    want[r0:r0 + 2, c0:c0 + 2] = blk
                    enc = Z.compress(np.ascontiguousarray(blk).tobytes())
                    index += [len(body), len(enc)]
                    body += enc
            ib = struct.pack("<%dQ" % len(index), *index)
            ib += struct.pack("<I", zlib.crc32(ib))                   # checksum bytes (not verified)
            fp = path / "c" / str(si) / str(sj)
            os.makedirs(fp.parent, exist_ok=True)
            fp.write_bytes(body + ib)
    assert np.array_equal(O.read_zarr3(str(path)), want)
