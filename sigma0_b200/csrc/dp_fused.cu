// Fused data-parallel gradient sync + AdamW for sm_100a over NVLink peer memory.
//
// One cooperative kernel per rank replaces "NCCL reduce-scatter -> norm
// all-reduce -> Adam on the shard -> NCCL all-gather" (the reference's pmean
// over `data`, src/base_model/training/train_helpers.py:2123-2196, plus its
// optax update).  Every rank's flat gradient, flat fp32 parameters and bf16
// shadow live in symmetric (peer-mapped) buffers; rank r owns the flat slice
// [lo, hi) and:
//   phase 0  waits until every peer's gradient is complete (flag exchange);
//   phase 1  sums its slice of all peers' gradients with float4 peer loads,
//            scales by 1/world, keeps the result in its own gradient slice and
//            accumulates the slice's sum of squares;
//   phase 2  exchanges the partial sums of squares (peer stores + flags), so
//            every rank has the global gradient norm for clipping;
//   phase 3  runs AdamW on the slice and stores the new fp32 parameters and
//            bf16 shadow straight into every peer's buffers (peer stores), then
//            signals completion; the next forward starts only after all peers'
//            slices have arrived.
// All cross-GPU waits are bounded spins: on timeout the kernel records the
// phase in `status`, still meets every grid barrier, and returns, so the host
// can raise instead of hanging.  Loads and stores to peers are plain global
// accesses (no TMA, no multicast).
#include <cooperative_groups.h>

#include "common.cuh"
#include "launchers.h"

namespace cg = cooperative_groups;

namespace s0 {
namespace dpf {

constexpr int NT = 256;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-rank barrier for `phase`, run by block 0 (its first `world` threads
// signal and wait).  Sets *abort and the status word when a peer's flag does
// not arrive within spin_limit polls.
__device__ void xbar(const DpfArgs& a, int phase, int* abort) {
  const int t = threadIdx.x;
  __threadfence_system();
  __syncthreads();
  if (t < a.world) {
    if (t != a.rank) st_release_sys(a.flags[t] + phase * DPF_MAXW + a.rank, a.seq);
    const int* mine = a.flags[a.rank] + phase * DPF_MAXW + t;
    if (t != a.rank) {
      long long it = 0;
      while (ld_acquire_sys(mine) < a.seq) {
        if (++it > a.spin_limit) {
          atomicExch(abort, 1);
          atomicExch(a.status, 100 + phase);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(NT) dp_fused_adam(DpfArgs a) {
  cg::grid_group grid = cg::this_grid();
  __shared__ float red[NT / 32];
  const long n4 = (a.hi - a.lo) / 4;
  const long tid = (long)blockIdx.x * NT + threadIdx.x, nthr = (long)gridDim.x * NT;
  // phase 0: all gradients complete
  if (blockIdx.x == 0) xbar(a, 0, a.abort);
  grid.sync();
  if (*((volatile int*)a.abort)) return;
  // phase 1: reduce this rank's slice over peers
  float ss = 0.f;
  float4* own = reinterpret_cast<float4*>(a.G[a.rank] + a.lo);
  for (long j = tid; j < n4; j += nthr) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < a.world; ++k) {
      const float4 g = reinterpret_cast<const float4*>(a.G[k] + a.lo)[j];
      acc.x += g.x; acc.y += g.y; acc.z += g.z; acc.w += g.w;
    }
    acc.x *= a.inv_world; acc.y *= a.inv_world; acc.z *= a.inv_world; acc.w *= a.inv_world;
    own[j] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < NT / 32; ++w) t += red[w];
    atomicAdd(a.sumsq_local, t);
  }
  grid.sync();
  // phase 2: global sum of squares
  if (blockIdx.x == 0) {
    if (threadIdx.x < a.world) a.sums[threadIdx.x][a.rank] = *((volatile float*)a.sumsq_local);
    xbar(a, 1, a.abort);
  }
  grid.sync();
  if (*((volatile int*)a.abort)) return;
  float total = 0.f;
  for (int k = 0; k < a.world; ++k) total += ((volatile float*)a.sums[a.rank])[k];
  float scale = 1.f;
  if (a.max_norm > 0.f) {
    const float nrm = sqrtf(total);
    scale = nrm < a.max_norm ? 1.f : a.max_norm / nrm;
  }
  // phase 3: AdamW on the slice, new values pushed to every rank
  for (long j = tid; j < n4; j += nthr) {
    const long i0 = a.lo + 4 * j;
    const bool ssm = i0 < a.n_ssm;   // group boundaries are multiples of 128
    const float lr = ssm ? a.lr_s : a.lr_r, wd = ssm ? 0.f : a.wd;
    const float4 g4 = own[j];
    float4 m4 = reinterpret_cast<float4*>(a.m)[j], v4 = reinterpret_cast<float4*>(a.v)[j];
    float4 p4 = reinterpret_cast<const float4*>(a.P[a.rank] + a.lo)[j];
    float* mp = &m4.x;
    float* vp = &v4.x;
    float* pp = &p4.x;
    const float* gg = &g4.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gi = gg[e] * scale;
      const float mi = a.b1 * mp[e] + (1.f - a.b1) * gi;
      const float vi = a.b2 * vp[e] + (1.f - a.b2) * gi * gi;
      mp[e] = mi;
      vp[e] = vi;
      const float upd = (mi / a.bc1) / (sqrtf(vi / a.bc2) + a.eps) + wd * pp[e];
      pp[e] -= lr * upd;
    }
    reinterpret_cast<float4*>(a.m)[j] = m4;
    reinterpret_cast<float4*>(a.v)[j] = v4;
    const uint2 sb = make_uint2(pack_bf16(p4.x, p4.y), pack_bf16(p4.z, p4.w));
    for (int k = 0; k < a.world; ++k) {
      const int kk = (a.rank + k) % a.world;   // stagger targets across ranks
      reinterpret_cast<float4*>(a.P[kk] + a.lo)[j] = p4;
      if (a.S[kk]) reinterpret_cast<uint2*>(a.S[kk] + a.lo)[j] = sb;
    }
  }
  grid.sync();
  // phase 4: every slice delivered everywhere
  if (blockIdx.x == 0) xbar(a, 2, a.abort);
}

}  // namespace dpf
}  // namespace s0

int dp_fused_adam_launch(const DpfArgs& a, int sms, cudaStream_t st) {
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s0::dpf::dp_fused_adam, s0::dpf::NT, 0);
  if (per_sm < 1) return -1;
  const long n4 = (a.hi - a.lo) / 4;
  long want = (n4 + s0::dpf::NT - 1) / s0::dpf::NT;
  long cap = (long)sms * (per_sm < 4 ? per_sm : 4);
  int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
  DpfArgs args = a;
  void* kargs[] = {&args};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)s0::dpf::dp_fused_adam, dim3(grid), dim3(s0::dpf::NT),
                                              kargs, 0, st);
  return e == cudaSuccess ? 0 : (int)e;
}
