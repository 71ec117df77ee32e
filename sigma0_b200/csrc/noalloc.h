// C entry point of the RMSNorm backward that allocates no device memory.
//
// This entry point has no counterpart in the reference.  It is for callers that
// cannot allocate device memory: a C or C++ host runtime that loads this
// library through its C ABI (dlopen, ctypes) without PyTorch's caching
// allocator, typically while a serving pool has already reserved the free HBM
// for recurrent state.  There a cudaMalloc would fail, or would synchronise the
// device in the middle of a pipelined step.  The outputs equal those of the
// tensor entry point `rms_bwd` (dw up to float summation order).
//
// Scratch: one file-scope device array of S0_NOALLOC_SCRATCH_BYTES (about
// 1.2 MB), which every GPU that loads the library holds until the process
// exits.  All calls on a device share it, and it keeps the last call's
// contents.  Calls that overlap on the GPU (two streams, or two host threads
// without ordering) race on it: the caller must serialise them.
// The first call on a device resolves the array's device address
// (cudaGetSymbolAddress) and sets a kernel attribute; make that first call
// before any stream capture on that device.
// Limits: D (row width) a multiple of 8 and at most S0_NOALLOC_MAX_D;
// 1 <= T (rows) <= 2^31 - 1; dy, x and dx start on a 16-byte boundary (rows are
// moved 16 bytes at a time).
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define S0_NOALLOC_MAX_D 2048
#define S0_NOALLOC_MAX_PARTS 148
#define S0_NOALLOC_SCRATCH_BYTES (S0_NOALLOC_MAX_PARTS * S0_NOALLOC_MAX_D * 4 + 256)

// dy, x, dx: bf16 [T, D]; w: fp32 [D]; rstd: fp32 [T] (from the forward);
// dw: fp32 [D], overwritten (it need not be zeroed).  `stream` is a
// cudaStream_t (NULL = the legacy default stream).  Returns 0 on success, -1
// when an argument is out of range, or the cudaError_t of a failed CUDA call;
// s0_noalloc_last_error() then describes the failure (per host thread).
int s0_rms_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                       long long T, int D, void* stream);
const char* s0_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
