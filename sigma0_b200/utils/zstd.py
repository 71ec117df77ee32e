"""Zstandard through the system's ``libzstd`` (ctypes), for images without the ``zstandard``
Python module.

The reference stores its LOBSTER day arrays as ``.npy.zst`` and Orbax can write zarr chunks
with the zstd codec; both are read here with this wrapper when ``zstandard`` is not
installed.  ``decompress`` handles frames with and without a recorded content size (the
latter through the streaming API) and concatenated frames; ``compress`` writes one frame
(tests, writers).
"""
from __future__ import annotations

import ctypes
import ctypes.util
from typing import Optional

_LIB = None
_CONTENTSIZE_UNKNOWN = (1 << 64) - 1
_CONTENTSIZE_ERROR = (1 << 64) - 2


class ZstdError(RuntimeError):
    pass


class _InBuf(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("size", ctypes.c_size_t), ("pos", ctypes.c_size_t)]


class _OutBuf(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("size", ctypes.c_size_t), ("pos", ctypes.c_size_t)]


def _lib():
    global _LIB
    if _LIB is None:
        name = ctypes.util.find_library("zstd") or "libzstd.so.1"
        try:
            lib = ctypes.CDLL(name)
        except OSError as e:
            raise ZstdError(f"libzstd is not available ({e}); install the zstandard module") from e
        lib.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
        lib.ZSTD_getFrameContentSize.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        lib.ZSTD_decompress.restype = ctypes.c_size_t
        lib.ZSTD_decompress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        lib.ZSTD_compress.restype = ctypes.c_size_t
        lib.ZSTD_compress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_int]
        lib.ZSTD_compressBound.restype = ctypes.c_size_t
        lib.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
        lib.ZSTD_isError.restype = ctypes.c_uint
        lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
        lib.ZSTD_getErrorName.restype = ctypes.c_char_p
        lib.ZSTD_getErrorName.argtypes = [ctypes.c_size_t]
        lib.ZSTD_createDStream.restype = ctypes.c_void_p
        lib.ZSTD_freeDStream.argtypes = [ctypes.c_void_p]
        lib.ZSTD_initDStream.restype = ctypes.c_size_t
        lib.ZSTD_initDStream.argtypes = [ctypes.c_void_p]
        lib.ZSTD_decompressStream.restype = ctypes.c_size_t
        lib.ZSTD_decompressStream.argtypes = [ctypes.c_void_p, ctypes.POINTER(_OutBuf), ctypes.POINTER(_InBuf)]
        lib.ZSTD_DStreamOutSize.restype = ctypes.c_size_t
        _LIB = lib
    return _LIB


def available() -> bool:
    try:
        _lib()
        return True
    except ZstdError:
        return False


def _check(lib, code: int, what: str) -> int:
    if lib.ZSTD_isError(code):
        raise ZstdError(f"{what}: {lib.ZSTD_getErrorName(code).decode()}")
    return code


def decompress(data: bytes, max_output: Optional[int] = None) -> bytes:
    """All frames of ``data`` decompressed and concatenated."""
    lib = _lib()
    src = ctypes.create_string_buffer(bytes(data), len(data))
    size = lib.ZSTD_getFrameContentSize(src, len(data))
    if size == _CONTENTSIZE_ERROR:
        raise ZstdError("not a zstd frame")
    if size != _CONTENTSIZE_UNKNOWN and (max_output is None or size <= max_output):
        # one frame of known size: one call (a following frame makes the size check fail
        # and falls back to streaming)
        dst = ctypes.create_string_buffer(max(int(size), 1))
        n = lib.ZSTD_decompress(dst, int(size), src, len(data))
        if not lib.ZSTD_isError(n):
            return dst.raw[:n]
    ds = lib.ZSTD_createDStream()
    try:
        _check(lib, lib.ZSTD_initDStream(ds), "initDStream")
        chunk = int(lib.ZSTD_DStreamOutSize())
        out = ctypes.create_string_buffer(chunk)
        inb = _InBuf(ctypes.cast(src, ctypes.c_void_p), len(data), 0)
        parts = []
        total = 0
        while True:
            ob = _OutBuf(ctypes.cast(out, ctypes.c_void_p), chunk, 0)
            ret = _check(lib, lib.ZSTD_decompressStream(ds, ctypes.byref(ob), ctypes.byref(inb)), "decompress")
            parts.append(out.raw[:ob.pos])
            total += ob.pos
            if max_output is not None and total > max_output:
                raise ZstdError(f"output exceeds {max_output} bytes")
            if inb.pos >= inb.size and ob.pos < chunk:
                if ret != 0:
                    raise ZstdError("truncated zstd input")
                break
        return b"".join(parts)
    finally:
        lib.ZSTD_freeDStream(ds)


def compress(data: bytes, level: int = 3) -> bytes:
    lib = _lib()
    src = ctypes.create_string_buffer(bytes(data), len(data))
    cap = lib.ZSTD_compressBound(len(data))
    dst = ctypes.create_string_buffer(cap)
    n = _check(lib, lib.ZSTD_compress(dst, cap, src, len(data), level), "compress")
    return dst.raw[:n]
