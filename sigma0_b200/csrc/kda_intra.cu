// Intra-chunk score and WY matrices of Kimi Delta Attention (per-key-dim decay), for
// sm_100a.
//
// With a decay per key dimension the chunkwise delta rule (the reference's
// _chunkwise_gdn with per-dim alpha, src/base_model/models/gdn.py:449-617) needs, per
// chunk of C = 64 steps,
//
//   intra_ij = sum_d q_id  k_jd exp(G_id - G_jd)      (i >= j, else 0)
//   Lm_ij    = -sum_d kb_id k_jd exp(G_id - G_jd)     (i >  j, else 0)
//
// where G is the within-chunk cumulative log decay.  The weight depends on i, j and d
// together, so these are not matrix products; written as tensor expressions they
// materialise a [C, C, hd] weight per chunk (and more in the backward).  Here every
// weight is formed in registers from G (exp2 of a difference, never above 1) and
// consumed at once:
//   forward : one CTA per chunk, thread (i, 16 columns j), the key dim streamed through
//             shared memory in tiles of 32;
//   backward: one CTA per (chunk, 32 key dims), thread (d, rows i = s mod 8):
//             dq_id = sum_j gI_ij k_jd w,  dkb_id = -sum_j gL_ij k_jd w  (thread-local),
//             dk_jd = sum_i (gI_ij q_id - gL_ij kb_id) w  (shared-memory atomics),
//             dG = q dq + kb dkb - k dk  (w depends on G_id - G_jd).
#include <cuda_runtime.h>

#include "launchers.h"

namespace s0 {
namespace kda {

constexpr int C = 64, DT = 32, NT = 256;
constexpr float LOG2E = 1.4426950408889634f;

__global__ void __launch_bounds__(NT) kda_intra_fwd_k(KdaArgs a) {
  __shared__ float sq[C][DT + 1], sk[C][DT + 1], skb[C][DT + 1], sg[C][DT + 1];
  const long n = blockIdx.x;
  const int tid = threadIdx.x, i = tid >> 2, j0 = tid & 3, HD = a.HD;
  const float* q = a.q + n * C * HD;
  const float* k = a.k + n * C * HD;
  const float* kb = a.kb + n * C * HD;
  const float* G = a.G + n * C * HD;
  float ai[16], al[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) ai[m] = al[m] = 0.f;
  for (int d0 = 0; d0 < HD; d0 += DT) {
    __syncthreads();
    for (int e = tid; e < C * DT; e += NT) {
      const int r = e / DT, c = e % DT;
      const long gi = (long)r * HD + d0 + c;
      sq[r][c] = q[gi];
      sk[r][c] = k[gi];
      skb[r][c] = kb[gi];
      sg[r][c] = G[gi] * LOG2E;
    }
    __syncthreads();
#pragma unroll 4
    for (int d = 0; d < DT; ++d) {
      const float qi = sq[i][d], kbi = skb[i][d], gi = sg[i][d];
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int j = j0 + 4 * m;
        if (j <= i) {
          const float w = exp2f(gi - sg[j][d]) * sk[j][d];
          ai[m] = fmaf(qi, w, ai[m]);
          al[m] = fmaf(kbi, w, al[m]);
        }
      }
    }
  }
  float* I = a.intra + n * C * C + (long)i * C;
  float* L = a.Lm + n * C * C + (long)i * C;
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int j = j0 + 4 * m;
    I[j] = j <= i ? ai[m] : 0.f;
    L[j] = j < i ? -al[m] : 0.f;
  }
}

constexpr size_t BWD_SMEM = (5 * C * (DT + 1) + 2 * C * (C + 1)) * sizeof(float);   // 75.5 KB

__global__ void __launch_bounds__(NT) kda_intra_bwd_k(KdaArgs a) {
  extern __shared__ float smem[];
  auto sq = reinterpret_cast<float(*)[DT + 1]>(smem);
  auto sk = sq + C, skb = sk + C, sg = skb + C, sdk = sg + C;
  auto sgI = reinterpret_cast<float(*)[C + 1]>(smem + 5 * C * (DT + 1));
  auto sgL = sgI + C;
  const int HD = a.HD, ndt = HD / DT;
  const long n = blockIdx.x / ndt;
  const int d0 = (blockIdx.x % ndt) * DT;
  const int tid = threadIdx.x, d = tid & (DT - 1), s = tid >> 5;   // s: rows i = s, s + 8, ...
  const long base = n * C * HD;
  for (int e = tid; e < C * DT; e += NT) {
    const int r = e / DT, c = e % DT;
    const long gi = base + (long)r * HD + d0 + c;
    sq[r][c] = a.q[gi];
    sk[r][c] = a.k[gi];
    skb[r][c] = a.kb[gi];
    sg[r][c] = a.G[gi] * LOG2E;
    sdk[r][c] = 0.f;
  }
  for (int e = tid; e < C * C; e += NT) {
    const int r = e / C, c = e % C;
    sgI[r][c] = c <= r ? a.gI[n * C * C + e] : 0.f;
    sgL[r][c] = c < r ? a.gL[n * C * C + e] : 0.f;
  }
  __syncthreads();
  float dq[8], dkb[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i = s + 8 * u;
    const float qi = sq[i][d], kbi = skb[i][d], gi = sg[i][d];
    float aq = 0.f, ab = 0.f;
    for (int j = 0; j <= i; ++j) {
      const float w = exp2f(gi - sg[j][d]);
      const float kw = sk[j][d] * w;
      const float gI = sgI[i][j], gL = sgL[i][j];
      aq = fmaf(gI, kw, aq);
      ab = fmaf(gL, kw, ab);
      atomicAdd(&sdk[j][d], (gI * qi - gL * kbi) * w);
    }
    dq[u] = aq;
    dkb[u] = -ab;
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i = s + 8 * u;
    const long gi = base + (long)i * HD + d0 + d;
    const float dk = sdk[i][d];
    a.dq[gi] = dq[u];
    a.dkb[gi] = dkb[u];
    a.dk[gi] = dk;
    a.dG[gi] = sq[i][d] * dq[u] + skb[i][d] * dkb[u] - sk[i][d] * dk;
  }
}

}  // namespace kda
}  // namespace s0

int kda_intra_launch(const KdaArgs& a, bool bwd, cudaStream_t st) {
  using namespace s0::kda;
  if (a.HD % DT || a.N <= 0) return a.N == 0 ? 0 : -1;
  if (!bwd) {
    kda_intra_fwd_k<<<(unsigned)a.N, NT, 0, st>>>(a);
  } else {
    cudaFuncSetAttribute(kda_intra_bwd_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BWD_SMEM);
    kda_intra_bwd_k<<<(unsigned)(a.N * (a.HD / DT)), NT, BWD_SMEM, st>>>(a);
  }
  return (int)cudaGetLastError();
}
