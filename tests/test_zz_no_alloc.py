"""The allocation-free C entry point ``s0_rms_bwd_noalloc`` (csrc/noalloc.cu).

Some callers cannot allocate device memory -- a C/C++ runtime that drives this
library through its C ABI with no PyTorch allocator, while a pool has reserved
the free HBM.  This test calls the entry point the way such a caller would,
through its exported C symbol (ctypes), twice in a row on the same scratch, and
checks it against the tensor entry point ``rms_bwd``.  The file name makes
pytest collect it last, so a run stopping at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import sigma0_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.s0_rms_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.s0_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def _inputs(T, D, seed):
    from sigma0_b200.ops._ext import ext
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    w = 1.0 + 0.1 * torch.randn(D, device="cuda", generator=g)
    _, rstd = ext().rms_fwd(x, w, 1e-6)
    return dy, x, w, rstd


def _call(lib, dy, x, w, rstd, dx, dw):
    T, D = x.shape
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.s0_rms_bwd_noalloc(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                                dw.data_ptr(), T, D, st)
    assert rc == 0, lib.s0_noalloc_last_error().decode()


@pytest.mark.parametrize("T,D", [(4096, 2048), (1000, 512)])
def test_noalloc_rms_bwd_matches_tensor_entry_point(T, D):
    from sigma0_b200.ops._ext import ext
    lib = _lib()
    dx = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.full((D,), float("nan"), device="cuda")      # overwritten, not accumulated into
    for call, seed in enumerate((1, 2)):                     # two calls in a row share the scratch
        dy, x, w, rstd = _inputs(T, D, seed)
        torch.cuda.synchronize()
        alloc0 = torch.cuda.memory_allocated()
        free0 = torch.cuda.mem_get_info()[0]
        _call(lib, dy, x, w, rstd, dx, dw)
        torch.cuda.synchronize()
        if call == 1:   # after the first call's one-time set-up, no device memory changes hands
            assert torch.cuda.mem_get_info()[0] == free0
        assert torch.cuda.memory_allocated() == alloc0
        dx_ref, dw_ref = ext().rms_bwd(dy, x, w, rstd)
        torch.cuda.synchronize()
        assert torch.allclose(dx.float(), dx_ref.float(), rtol=1e-2, atol=1e-2)
        assert torch.allclose(dw, dw_ref, rtol=1e-4, atol=1e-3), (dw - dw_ref).abs().max()


def test_noalloc_rejects_oversized_rows():
    lib = _lib()
    D = 4096
    x = torch.zeros(8, D, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(D, device="cuda")
    r = torch.ones(8, device="cuda")
    dw = torch.zeros(D, device="cuda")
    rc = lib.s0_rms_bwd_noalloc(x.data_ptr(), x.data_ptr(), w.data_ptr(), r.data_ptr(), x.data_ptr(),
                                dw.data_ptr(), 8, D, None)
    assert rc == -1
    assert b"at most 2048" in lib.s0_noalloc_last_error()


def test_noalloc_rejects_misaligned_rows():
    """A buffer that starts 8 bytes past a 16-byte boundary is refused with -1, not read."""
    lib = _lib()
    D = 512
    buf = torch.zeros(8 * D + 8, device="cuda", dtype=torch.bfloat16)
    x = buf[4:4 + 8 * D]                  # 8-byte offset from the allocation's base
    assert x.data_ptr() % 16 == 8
    w = torch.ones(D, device="cuda")
    r = torch.ones(8, device="cuda")
    dw = torch.zeros(D, device="cuda")
    rc = lib.s0_rms_bwd_noalloc(x.data_ptr(), x.data_ptr(), w.data_ptr(), r.data_ptr(), x.data_ptr(),
                                dw.data_ptr(), 8, D, None)
    assert rc == -1
    assert b"16-byte aligned" in lib.s0_noalloc_last_error()
