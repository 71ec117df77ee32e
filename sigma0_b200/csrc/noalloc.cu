// RMSNorm backward without device allocation (declared in noalloc.h).
//
// Same math as rms_bwd_k in fused_ops.cu: dx = r*g*w - x*r^3*mean(g*w*x),
// dw = sum over rows of g*x*r.  The column sums for dw go through a static
// scratch array instead of an atomically accumulated, zero-initialised output:
//   1. each block reduces its rows' g*x*r per column and writes one partial
//      row into scratch.part[block][0..D);
//   2. it then draws a ticket from scratch.ticket; the block that draws the
//      last ticket sums the partial rows into dw (overwriting it) and puts the
//      ticket back to zero.
// Only the ticket must start at zero.  The array keeps the previous call's
// contents, so every call also clears the ticket with a 4-byte cudaMemsetAsync
// on its stream before the launch.
#include "common.cuh"
#include "noalloc.h"

#include <cstdint>
#include <cstdio>
#include <mutex>

namespace {

using bf16 = __nv_bfloat16;
using s0::pack_bf16;
using s0::unpack_bf16;
using s0::warp_sum;

constexpr int NT = 256;
constexpr int MAX_DEV = 64;

struct Scratch {
  unsigned int ticket;
  unsigned int pad[63];
  float part[S0_NOALLOC_MAX_PARTS * S0_NOALLOC_MAX_D];
};
static_assert(sizeof(Scratch) <= S0_NOALLOC_SCRATCH_BYTES, "scratch size");

static __device__ __align__(256) Scratch g_scratch;

template <int PER>
__global__ void __launch_bounds__(NT)
    rms_bwd_noalloc_k(const bf16* __restrict__ dy, const bf16* __restrict__ x, const float* __restrict__ w,
                      const float* __restrict__ rstd, bf16* __restrict__ dx, float* __restrict__ dw,
                      Scratch* __restrict__ sc, long long T, int D) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nwb = NT / 32;
  const long long gw = (blockIdx.x * NT + threadIdx.x) >> 5, nw = (gridDim.x * NT) >> 5;
  const int nv = D / 8;
  float aw[PER * 8];
#pragma unroll
  for (int i = 0; i < PER * 8; ++i) aw[i] = 0.f;
  // 64-bit row index: T may be close to 2^31 - 1, where row + nw would overflow an int
  for (long long row = gw; row < T; row += nw) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * D);
    const float r = rstd[row];
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        uint4 ux = xr[c], ug = gr[c];
        uint32_t ax[4] = {ux.x, ux.y, ux.z, ux.w}, ag[4] = {ug.x, ug.y, ug.z, ug.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          const int col = c * 8 + 2 * k;
          m += fg.x * w[col] * fx.x + fg.y * w[col + 1] * fx.y;
          aw[j * 8 + 2 * k] += fg.x * fx.x * r;
          aw[j * 8 + 2 * k + 1] += fg.y * fx.y * r;
        }
      }
    }
    m = warp_sum(m) / D;
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        uint4 ux = xr[c], ug = gr[c];
        uint32_t ax[4] = {ux.x, ux.y, ux.z, ux.w}, ag[4] = {ug.x, ug.y, ug.z, ug.w}, o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          const int col = c * 8 + 2 * k;
          o[k] = pack_bf16(r * fg.x * w[col] - fx.x * r * r * r * m, r * fg.y * w[col + 1] - fx.y * r * r * r * m);
        }
        dr[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // this block's partial of dw -> scratch row blockIdx.x
  extern __shared__ float red[];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int c = lane + 32 * j;
    if (c < nv)
#pragma unroll
      for (int k = 0; k < 8; ++k) red[wid * D + c * 8 + k] = aw[j * 8 + k];
  }
  __syncthreads();
  float* mine = sc->part + (size_t)blockIdx.x * D;
  for (int col = threadIdx.x; col < D; col += NT) {
    float t = 0.f;
    for (int k = 0; k < nwb; ++k) t += red[k * D + col];
    mine[col] = t;
  }
  // the last block to finish sums the partial rows
  __threadfence();
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&sc->ticket, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int col = threadIdx.x; col < D; col += NT) {
    float t = 0.f;
    for (int b = 0; b < (int)gridDim.x; ++b) t += __ldcg(sc->part + (size_t)b * D + col);
    dw[col] = t;
  }
  if (threadIdx.x == 0) sc->ticket = 0u;
}

// per-device set-up: the scratch's device address, resolved once with the device current
std::mutex g_mu;
bool g_ready[MAX_DEV];
Scratch* g_ptr[MAX_DEV];
thread_local char g_msg[256] = "no error";

int fail(int code, const char* what) {
  std::snprintf(g_msg, sizeof(g_msg), "%s", what);
  return code;
}

int setup(int dev, Scratch** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ready[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) {
      std::snprintf(g_msg, sizeof(g_msg), "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                    cudaGetErrorString(e));
      return (int)e;
    }
    const int smem = (NT / 32) * S0_NOALLOC_MAX_D * 4;
    e = cudaFuncSetAttribute(rms_bwd_noalloc_k<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      std::snprintf(g_msg, sizeof(g_msg), "cudaFuncSetAttribute failed on device %d: %s", dev,
                    cudaGetErrorString(e));
      return (int)e;
    }
    g_ptr[dev] = static_cast<Scratch*>(p);
    g_ready[dev] = true;
  }
  *out = g_ptr[dev];
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* s0_noalloc_last_error(void) { return g_msg; }

extern "C" __attribute__((visibility("default"))) int s0_rms_bwd_noalloc(const void* dy, const void* x,
                                                                          const float* w, const float* rstd,
                                                                          void* dx, float* dw, long long T, int D,
                                                                          void* stream) {
  if (D <= 0 || D % 8 != 0 || D > S0_NOALLOC_MAX_D) {
    std::snprintf(g_msg, sizeof(g_msg), "s0_rms_bwd_noalloc: D=%d must be a positive multiple of 8 and at most %d",
                  D, S0_NOALLOC_MAX_D);
    return -1;
  }
  if (T <= 0 || T > 2147483647LL) {
    std::snprintf(g_msg, sizeof(g_msg), "s0_rms_bwd_noalloc: T=%lld rows must be in [1, 2^31 - 1]", T);
    return -1;
  }
  if (!dy || !x || !w || !rstd || !dx || !dw) return fail(-1, "s0_rms_bwd_noalloc: null pointer argument");
  // rows of dy, x and dx are read and written 16 bytes at a time: their base addresses must be
  // 16-byte aligned (D % 8 == 0 keeps every row start aligned once the base is)
  if ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dx)) & 15u)
    return fail(-1, "s0_rms_bwd_noalloc: dy, x and dx must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail((int)e, "cudaGetDevice failed");
  if (dev < 0 || dev >= MAX_DEV) return fail(-1, "s0_rms_bwd_noalloc: device ordinal out of range");
  Scratch* sc = nullptr;
  const int rc = setup(dev, &sc);
  if (rc != 0) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(&sc->ticket, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return fail((int)e, "cudaMemsetAsync(ticket) failed");
  const long long want = (T + 7) / 8;
  const int blocks = (int)(want < S0_NOALLOC_MAX_PARTS ? want : S0_NOALLOC_MAX_PARTS);
  const int nv = D / 8;
  const size_t smem = (size_t)(NT / 32) * D * 4;
  const bf16* g = reinterpret_cast<const bf16*>(dy);
  const bf16* xp = reinterpret_cast<const bf16*>(x);
  bf16* o = reinterpret_cast<bf16*>(dx);
  if (nv <= 32) rms_bwd_noalloc_k<1><<<blocks, NT, smem, st>>>(g, xp, w, rstd, o, dw, sc, T, D);
  else if (nv <= 64) rms_bwd_noalloc_k<2><<<blocks, NT, smem, st>>>(g, xp, w, rstd, o, dw, sc, T, D);
  else if (nv <= 128) rms_bwd_noalloc_k<4><<<blocks, NT, smem, st>>>(g, xp, w, rstd, o, dw, sc, T, D);
  else rms_bwd_noalloc_k<8><<<blocks, NT, smem, st>>>(g, xp, w, rstd, o, dw, sc, T, D);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::snprintf(g_msg, sizeof(g_msg), "s0_rms_bwd_noalloc launch failed: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}
