// Causal / sliding-window flash attention, forward and backward, for sm_100a.
//
// Replaces the attention of the transformer, hybrid and NSA window branches (the
// reference calls cuDNN's flash attention, src/base_model/models/nsa.py:27-59, and a
// Pallas MHA, src/base_model/models/transformer.py:19-85).  Query i (absolute position
// q_offset + i) attends to keys j <= q_offset + i, and with a window W only to
// j > q_offset + i - W; keys beyond Lk do not exist.  Optional tables give every key its
// own absolute position (compressed or gathered key blocks: NSA) and every batch entry
// its own query offset (query groups flattened into the batch).  Layouts are the models' own:
// q/o [B, Lq, nh, HD], k/v [B, Lk, nh, HD] with arbitrary batch / row / head strides
// (elements; multiples of 8) and contiguous head dimension HD in {64, 128}.
//
// Forward  (grid: query blocks of 128 x heads x batch, 8 warps of 16 query rows):
//   Q fragments stay in registers; K/V blocks of 64 keys stream through a two-stage
//   cp.async ring; S = Q K^T and O += P V on bf16 tensor cores (mma.m16n8k16, fp32
//   accumulate); online softmax in the base-2 domain; O is normalised, staged through
//   shared memory and stored with 16-byte stores; the row log-sum-exp (base 2) is kept
//   for the backward.
// Backward (grid: key blocks of 128 x heads x batch, 8 warps of 16 keys):
//   the CTA walks the query blocks (64 rows) that see its keys; per block it recomputes
//   P^T = exp2(K Q^T * c - lse), accumulates dV += P^T dO and dK += dS^T Q in registers
//   (dS = P (dP - D), dP^T = V dO^T, D = rowsum(dO O)), stages dS^T in shared memory and
//   adds dQ = dS K into an fp32 buffer with vector atomics.  Masked blocks take the
//   per-element test, the others skip it.
#include <cuda_bf16.h>
#include <math_constants.h>

#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace attn {

using bf16 = __nv_bfloat16;
constexpr int NT = 256;

// key index `key` sits at absolute position `kp` (= key unless a position table is given)
__device__ __forceinline__ bool visible(int key, int kp, int qpos, int Lk, int window) {
  return key < Lk && kp <= qpos && (window <= 0 || kp > qpos - window);
}
__device__ __forceinline__ int key_pos(const int* kp, int key, int Lk) {
  return kp ? (key < Lk ? __ldg(kp + key) : 0x7fffffff) : key;
}

// rows x HD tile of a strided [.., rows, .., HD] tensor -> shared [rows][HD + 8], zero-filled
// past `nrows`
template <int HD>
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, long row_stride, int rows, int nrows, int tid) {
  constexpr int C = HD / 8;
  for (int i = tid; i < rows * C; i += NT) {
    const int r = i / C, c = i % C;
    const bool ok = r < nrows;
    cp_async16(s + r * (HD + 8) + c * 8, ok ? g + (long)r * row_stride + c * 8 : g, ok ? 16 : 0);
  }
}

// ------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------
template <int HD, bool SEL>
__global__ void __launch_bounds__(NT, HD == 64 ? 2 : 1) attn_fwd_k(AttnArgs a) {
  constexpr int BQ = 128, BKV = 64, LDS = HD + 8, KS = HD / 16;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem);
  bf16* sK = sQ + BQ * LDS;                     // [2][BKV][LDS]
  bf16* sV = sK + 2 * BKV * LDS;                // [2][BKV][LDS]
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const bf16* qg = a.q + b * a.sq_b + (long)q0 * a.sq_l + h * a.sq_h;
  const long kb_b = SEL ? (long)(b / a.kb_ng) : (long)b;             // the batch the keys come from
  const bf16* kg = a.k + kb_b * a.sk_b + h * a.sk_h;
  const bf16* vg = a.v + kb_b * a.sv_b + h * a.sv_h;
  // first source row of logical key block j (64 keys; block-indirect with SEL)
  auto krow = [&](int j) -> long {
    if constexpr (SEL) return (long)min(max(__ldg(a.kblk + (long)b * a.kb_n + j), 0), a.kb_max) * BKV;
    else return (long)j * BKV;
  };
  const int qoff = a.qoff ? a.qoff[b] : a.q_offset;
  const int* kp = a.kpos ? a.kpos + (long)b * a.Lk : nullptr;     // per-key positions (else the index)
  const int qlo = qoff + q0;                                         // smallest query position here
  int kb0 = 0, kb1 = (a.Lk + BKV - 1) / BKV;
  if (!kp) {
    const int hi = min(a.Lk, qlo + BQ);                              // keys [lo, hi) can be visible
    const int lo = a.window > 0 ? max(0, qlo - a.window + 1) : 0;
    kb0 = lo / BKV;
    kb1 = (hi + BKV - 1) / BKV;
  }

  load_tile<HD>(sQ, qg, a.sq_l, BQ, a.Lq - q0, tid);
  if (kb0 < kb1) {
    load_tile<HD>(sK, kg + krow(kb0) * a.sk_l, a.sk_l, BKV, a.Lk - kb0 * BKV, tid);
    load_tile<HD>(sV, vg + krow(kb0) * a.sv_l, a.sv_l, BKV, a.Lk - kb0 * BKV, tid);
  }
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-CUDART_INF_F, -CUDART_INF_F}, l[2] = {0.f, 0.f};
  uint32_t qf[KS][4];
  const int row0 = q0 + warp * 16 + g;                               // this thread's rows: row0, row0 + 8
  const int qp0 = qoff + row0, qp1 = qp0 + 8;

  for (int kb = kb0; kb < kb1; ++kb) {
    const int st = (kb - kb0) & 1;
    if (kb + 1 < kb1) {
      const int n = (kb + 1) * BKV;
      load_tile<HD>(sK + (st ^ 1) * BKV * LDS, kg + krow(kb + 1) * a.sk_l, a.sk_l, BKV, a.Lk - n, tid);
      load_tile<HD>(sV + (st ^ 1) * BKV * LDS, vg + krow(kb + 1) * a.sv_l, a.sv_l, BKV, a.Lk - n, tid);
    }
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    if (kb == kb0) {
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) load_a(qf[kk], sQ, LDS, warp * 16, kk * 16, lane);
    }
    const bf16* cK = sK + st * BKV * LDS;
    const bf16* cV = sV + st * BKV * LDS;
    float s[BKV / 8][4];
#pragma unroll
    for (int i = 0; i < BKV / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
#pragma unroll
      for (int np = 0; np < BKV / 16; ++np) {
        uint32_t bb[4];
        load_b_nk(bb, cK, LDS, np * 16, kk * 16, lane);
        mma_bf16(s[2 * np], qf[kk], bb[0], bb[1]);
        mma_bf16(s[2 * np + 1], qf[kk], bb[2], bb[3]);
      }
    // scale into the base-2 domain; per-element mask only where the block needs it
    const int key0 = kb * BKV;
    const bool full = !kp && key0 + BKV - 1 <= qlo && key0 + BKV <= a.Lk &&
                      (a.window <= 0 || key0 > qlo + BQ - 1 - a.window);
#pragma unroll
    for (int nt = 0; nt < BKV / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[nt][e] * a.scale_log2;
        if (!full) {
          const int key = key0 + nt * 8 + 2 * t + (e & 1);
          if (!visible(key, key_pos(kp, key, a.Lk), e < 2 ? qp0 : qp1, a.Lk, a.window)) x = -CUDART_INF_F;
        }
        s[nt][e] = x;
      }
    float mx[2] = {m[0], m[1]};
#pragma unroll
    for (int nt = 0; nt < BKV / 8; ++nt) {
      mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], base[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      base[r] = mx[r] == -CUDART_INF_F ? 0.f : mx[r];                 // a row with nothing visible yet
      alpha[r] = exp2f(m[r] - base[r]);
      m[r] = mx[r];
      l[r] *= alpha[r];
    }
#pragma unroll
    for (int nt = 0; nt < BKV / 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - base[0]);
      s[nt][1] = exp2f(s[nt][1] - base[0]);
      s[nt][2] = exp2f(s[nt][2] - base[1]);
      s[nt][3] = exp2f(s[nt][3] - base[1]);
      l[0] += s[nt][0] + s[nt][1];
      l[1] += s[nt][2] + s[nt][3];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t pa[4];
      acc_to_a(pa, s[2 * kk], s[2 * kk + 1]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t bb[4];
        load_b_kn(bb, cV, LDS, dp * 16, kk * 16, lane);
        mma_bf16(o[2 * dp], pa, bb[0], bb[1]);
        mma_bf16(o[2 * dp + 1], pa, bb[2], bb[3]);
      }
    }
    __syncthreads();                                                 // stage st free for the next prefetch
  }
  cp_async_wait_group<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  const float inv0 = l[0] > 0.f ? 1.f / l[0] : 0.f, inv1 = l[1] > 0.f ? 1.f / l[1] : 0.f;
  // stage the normalised rows (the Q tile is no longer read) and store them coalesced
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) {
    const int c = nt * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(sQ + (warp * 16 + g) * LDS + c) = pack_bf16(o[nt][0] * inv0, o[nt][1] * inv0);
    *reinterpret_cast<uint32_t*>(sQ + (warp * 16 + g + 8) * LDS + c) = pack_bf16(o[nt][2] * inv1, o[nt][3] * inv1);
  }
  if (t == 0) {
    float* lse = a.lse + ((long)b * a.nh + h) * a.Lq;
    // a row that saw no key gets +inf, so the backward's exp2(s - lse) is 0 there
    if (row0 < a.Lq) lse[row0] = l[0] > 0.f ? m[0] + log2f(l[0]) : CUDART_INF_F;
    if (row0 + 8 < a.Lq) lse[row0 + 8] = l[1] > 0.f ? m[1] + log2f(l[1]) : CUDART_INF_F;
  }
  __syncthreads();
  bf16* og = a.o + b * a.so_b + (long)q0 * a.so_l + h * a.so_h;
  constexpr int C = HD / 8;
  for (int i = tid; i < BQ * C; i += NT) {
    const int r = i / C, c = i % C;
    if (q0 + r < a.Lq)
      *reinterpret_cast<uint4*>(og + (long)r * a.so_l + c * 8) = *reinterpret_cast<const uint4*>(sQ + r * LDS + c * 8);
  }
}

// ------------------------------------------------------------------------------------------
// head-summed probabilities (NSA block importance; no gradient)
// ------------------------------------------------------------------------------------------
// imp[b, i, j] = sum_h exp2(s_bhij * c - lse_bhi) over visible keys: grid (query blocks of
// 128, key blocks of 64, batch); the heads stream through a two-stage ring of Q / K tiles
// and the sum stays in registers.  Tiles whose keys all lie after the last query are zero.
template <int HD>
__global__ void __launch_bounds__(NT) attn_probsum_k(AttnArgs a, float* imp) {
  constexpr int BQ = 128, BKV = 64, LDS = HD + 8, KS = HD / 16;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem);     // [2][BQ][LDS]
  bf16* sK = sQ + 2 * BQ * LDS;                 // [2][BKV][LDS]
  __shared__ int s_minpos;
  const int q0 = blockIdx.x * BQ, key0 = blockIdx.y * BKV, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int qoff = a.qoff ? a.qoff[b] : a.q_offset;
  const int* kp = a.kpos ? a.kpos + (long)b * a.Lk : nullptr;
  const int row0 = q0 + warp * 16 + g, qp0 = qoff + row0, qp1 = qp0 + 8;
  if (warp == 0) {
    int m = min(key_pos(kp, key0 + lane, a.Lk), key_pos(kp, key0 + 32 + lane, a.Lk));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_minpos = m;
  }
  __syncthreads();
  const bool any = s_minpos <= qoff + q0 + BQ - 1;
  float acc[BKV / 8][4];
#pragma unroll
  for (int i = 0; i < BKV / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  if (any) {
    auto load = [&](int h, int st) {
      load_tile<HD>(sQ + st * BQ * LDS, a.q + b * a.sq_b + (long)q0 * a.sq_l + h * a.sq_h, a.sq_l, BQ, a.Lq - q0, tid);
      load_tile<HD>(sK + st * BKV * LDS, a.k + b * a.sk_b + (long)key0 * a.sk_l + h * a.sk_h, a.sk_l, BKV,
                    a.Lk - key0, tid);
    };
    load(0, 0);
    cp_async_commit();
    for (int h = 0; h < a.nh; ++h) {
      const int st = h & 1;
      if (h + 1 < a.nh) load(h + 1, st ^ 1);
      cp_async_commit();
      cp_async_wait_group<1>();
      __syncthreads();
      const bf16* cQ = sQ + st * BQ * LDS;
      const bf16* cK = sK + st * BKV * LDS;
      float s[BKV / 8][4];
#pragma unroll
      for (int i = 0; i < BKV / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t qa[4];
        load_a(qa, cQ, LDS, warp * 16, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < BKV / 16; ++np) {
          uint32_t bb[4];
          load_b_nk(bb, cK, LDS, np * 16, kk * 16, lane);
          mma_bf16(s[2 * np], qa, bb[0], bb[1]);
          mma_bf16(s[2 * np + 1], qa, bb[2], bb[3]);
        }
      }
      const float* lse = a.lse + ((long)b * a.nh + h) * a.Lq;
      const float l0 = row0 < a.Lq ? lse[row0] : CUDART_INF_F, l1 = row0 + 8 < a.Lq ? lse[row0 + 8] : CUDART_INF_F;
#pragma unroll
      for (int nt = 0; nt < BKV / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + nt * 8 + 2 * t + (e & 1);
          const bool ok = visible(key, key_pos(kp, key, a.Lk), e < 2 ? qp0 : qp1, a.Lk, a.window);
          acc[nt][e] += ok ? exp2f(s[nt][e] * a.scale_log2 - (e < 2 ? l0 : l1)) : 0.f;
        }
      __syncthreads();                                               // stage st free
    }
    cp_async_wait_group<0>();
  }
  float* out = imp + (long)b * a.Lq * a.Lk;
#pragma unroll
  for (int nt = 0; nt < BKV / 8; ++nt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = row0 + 8 * hf, key = key0 + nt * 8 + 2 * t;
      if (row < a.Lq) {
        if (key < a.Lk) out[(long)row * a.Lk + key] = acc[nt][2 * hf];
        if (key + 1 < a.Lk) out[(long)row * a.Lk + key + 1] = acc[nt][2 * hf + 1];
      }
    }
}

// ------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------
// D[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d] (one warp per row)
template <int HD>
__global__ void __launch_bounds__(NT) attn_bwd_pre_k(AttnBwdArgs a) {
  const int w = (blockIdx.x * NT + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long rows = (long)a.f.B * a.f.nh * a.f.Lq;
  if (w >= rows) return;
  const int i = (int)(w % a.f.Lq), h = (int)((w / a.f.Lq) % a.f.nh), b = (int)(w / ((long)a.f.Lq * a.f.nh));
  const bf16* o = a.f.o + b * a.f.so_b + (long)i * a.f.so_l + h * a.f.so_h;
  const bf16* d = a.dout + b * a.sd_b + (long)i * a.sd_l + h * a.sd_h;
  float acc = 0.f;
  for (int c = lane * 2; c < HD; c += 64) {
    const float2 x = unpack_bf16(*reinterpret_cast<const uint32_t*>(o + c));
    const float2 y = unpack_bf16(*reinterpret_cast<const uint32_t*>(d + c));
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) a.D[w] = acc;
}

template <int HD>
__global__ void __launch_bounds__(NT, 1) attn_bwd_k(AttnBwdArgs a) {
  constexpr int BC = 128, BR = 64, LDS = HD + 8, KS = HD / 16, LDT = BR + 8;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sK = reinterpret_cast<bf16*>(smem);     // [BC][LDS]
  bf16* sV = sK + BC * LDS;                     // [BC][LDS]
  bf16* sQ = sV + BC * LDS;                     // [2][BR][LDS]
  bf16* sD = sQ + 2 * BR * LDS;                 // dO: [2][BR][LDS]
  bf16* sT = sD + 2 * BR * LDS;                 // dS^T: [BC][LDT]
  float* sL = reinterpret_cast<float*>(sT + BC * LDT);   // lse: [2][BR]
  float* sDD = sL + 2 * BR;                               // D:   [2][BR]
  const AttnArgs& f = a.f;
  const int k0 = blockIdx.x * BC, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const bf16* qg = f.q + b * f.sq_b + h * f.sq_h;
  const bf16* dg = a.dout + b * a.sd_b + h * a.sd_h;
  const float* lg = f.lse + ((long)b * f.nh + h) * f.Lq;
  const float* Dg = a.D + ((long)b * f.nh + h) * f.Lq;
  // query rows that can see keys [k0, k0 + BC)
  const int qoff = f.qoff ? f.qoff[b] : f.q_offset;
  const int* kp = f.kpos ? f.kpos + (long)b * f.Lk : nullptr;
  int qb0 = 0, qb1 = (f.Lq + BR - 1) / BR;
  if (!kp) {
    const int ilo = max(0, k0 - qoff);
    const int ihi = f.window > 0 ? min(f.Lq, k0 + BC - 1 + f.window - qoff) : f.Lq;
    qb0 = ilo / BR;
    qb1 = ihi > ilo ? (ihi + BR - 1) / BR : qb0;
  }

  if (f.kblk) {
    // block-indirect keys: the tile's two 64-key halves come from their own source blocks
    const long kb_b = (long)(b / f.kb_ng);
    const bf16* ks = f.k + kb_b * f.sk_b + h * f.sk_h;
    const bf16* vs = f.v + kb_b * f.sv_b + h * f.sv_h;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int j = blockIdx.x * 2 + half;
      const bool ok = j < f.kb_n;
      const long row = ok ? (long)min(max(__ldg(f.kblk + (long)b * f.kb_n + j), 0), f.kb_max) * (BC / 2) : 0;
      load_tile<HD>(sK + half * (BC / 2) * LDS, ks + row * f.sk_l, f.sk_l, BC / 2, ok ? BC / 2 : 0, tid);
      load_tile<HD>(sV + half * (BC / 2) * LDS, vs + row * f.sv_l, f.sv_l, BC / 2, ok ? BC / 2 : 0, tid);
    }
  } else {
    load_tile<HD>(sK, f.k + b * f.sk_b + (long)k0 * f.sk_l + h * f.sk_h, f.sk_l, BC, f.Lk - k0, tid);
    load_tile<HD>(sV, f.v + b * f.sv_b + (long)k0 * f.sv_l + h * f.sv_h, f.sv_l, BC, f.Lk - k0, tid);
  }
  auto load_q = [&](int qb, int st) {
    const int r0 = qb * BR;
    load_tile<HD>(sQ + st * BR * LDS, qg + (long)r0 * f.sq_l, f.sq_l, BR, f.Lq - r0, tid);
    load_tile<HD>(sD + st * BR * LDS, dg + (long)r0 * a.sd_l, a.sd_l, BR, f.Lq - r0, tid);
    if (tid < BR) {
      const bool ok = r0 + tid < f.Lq;
      cp_async4(sL + st * BR + tid, ok ? lg + r0 + tid : lg, ok ? 4 : 0);
      cp_async4(sDD + st * BR + tid, ok ? Dg + r0 + tid : Dg, ok ? 4 : 0);
    }
  };
  if (qb0 < qb1) load_q(qb0, 0);
  cp_async_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const int key_a = k0 + warp * 16 + g, key_b = key_a + 8;           // this thread's key rows
  const int kpa = key_pos(kp, key_a, f.Lk), kpb = key_pos(kp, key_b, f.Lk);
  const int kmax = k0 + BC - 1;

  for (int qb = qb0; qb < qb1; ++qb) {
    const int st = (qb - qb0) & 1;
    if (qb + 1 < qb1) load_q(qb + 1, st ^ 1);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    const bf16* cQ = sQ + st * BR * LDS;
    const bf16* cD = sD + st * BR * LDS;
    const float* cL = sL + st * BR;
    const float* cDD = sDD + st * BR;
    const int r0 = qb * BR;
    // S^T = K Q^T and dP^T = V dO^T for this warp's 16 keys x 64 queries
    float s[BR / 8][4], dp[BR / 8][4];
#pragma unroll
    for (int i = 0; i < BR / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t ka[4], va[4];
      load_a(ka, sK, LDS, warp * 16, kk * 16, lane);
      load_a(va, sV, LDS, warp * 16, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < BR / 16; ++np) {
        uint32_t bq[4], bd[4];
        load_b_nk(bq, cQ, LDS, np * 16, kk * 16, lane);
        load_b_nk(bd, cD, LDS, np * 16, kk * 16, lane);
        mma_bf16(s[2 * np], ka, bq[0], bq[1]);
        mma_bf16(s[2 * np + 1], ka, bq[2], bq[3]);
        mma_bf16(dp[2 * np], va, bd[0], bd[1]);
        mma_bf16(dp[2 * np + 1], va, bd[2], bd[3]);
      }
    }
    // P^T and dS^T (rows: keys key_a / key_b; columns: queries)
    const int qlo = qoff + r0, qhi = qlo + BR - 1;
    const bool full = !kp && kmax <= qlo && kmax < f.Lk && r0 + BR <= f.Lq && (f.window <= 0 || k0 > qhi - f.window);
#pragma unroll
    for (int nt = 0; nt < BR / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ci = nt * 8 + 2 * t + (e & 1);                    // query column within the block
        float p = exp2f(s[nt][e] * f.scale_log2 - cL[ci]);
        if (!full) {
          const int qi = r0 + ci;
          if (qi >= f.Lq || !(e < 2 ? visible(key_a, kpa, qoff + qi, f.Lk, f.window)
                                    : visible(key_b, kpb, qoff + qi, f.Lk, f.window)))
            p = 0.f;
        }
        s[nt][e] = p;
        dp[nt][e] = p * (dp[nt][e] - cDD[ci]);
      }
    // dV += P^T dO,  dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BR / 16; ++kk) {
      uint32_t pa[4], sa[4];
      acc_to_a(pa, s[2 * kk], s[2 * kk + 1]);
      acc_to_a(sa, dp[2 * kk], dp[2 * kk + 1]);
#pragma unroll
      for (int dpi = 0; dpi < HD / 16; ++dpi) {
        uint32_t bd[4], bq[4];
        load_b_kn(bd, cD, LDS, dpi * 16, kk * 16, lane);
        load_b_kn(bq, cQ, LDS, dpi * 16, kk * 16, lane);
        mma_bf16(dv[2 * dpi], pa, bd[0], bd[1]);
        mma_bf16(dv[2 * dpi + 1], pa, bd[2], bd[3]);
        mma_bf16(dk[2 * dpi], sa, bq[0], bq[1]);
        mma_bf16(dk[2 * dpi + 1], sa, bq[2], bq[3]);
      }
    }
    // dS^T -> shared (bf16, [key][query]) for the dQ product over all 128 keys
#pragma unroll
    for (int nt = 0; nt < BR / 8; ++nt) {
      const int c = nt * 8 + 2 * t;
      *reinterpret_cast<uint32_t*>(sT + (warp * 16 + g) * LDT + c) = pack_bf16(dp[nt][0], dp[nt][1]);
      *reinterpret_cast<uint32_t*>(sT + (warp * 16 + g + 8) * LDT + c) = pack_bf16(dp[nt][2], dp[nt][3]);
    }
    __syncthreads();
    // dQ[rows (w & 3) * 16 .. +16, cols (w >> 2) * HD/2 .. + HD/2] = dS K over the 128 keys
    {
      constexpr int NQ = HD / 2 / 8;
      const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * (HD / 2);
      float dq[NQ][4];
#pragma unroll
      for (int i = 0; i < NQ; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BC / 16; ++kk) {
        uint32_t aa[4];
        load_a_t(aa, sT, LDT, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < NQ / 2; ++np) {
          uint32_t bk[4];
          load_b_kn(bk, sK, LDS, n0 + np * 16, kk * 16, lane);
          mma_bf16(dq[2 * np], aa, bk[0], bk[1]);
          mma_bf16(dq[2 * np + 1], aa, bk[2], bk[3]);
        }
      }
      const int qa = r0 + m0 + g, qc = qa + 8;
      float* base = a.dq_acc + ((long)b * f.Lq * f.nh + h) * HD;       // [B, Lq, nh, HD] fp32
#pragma unroll
      for (int nt = 0; nt < NQ; ++nt) {
        const int c = n0 + nt * 8 + 2 * t;
        if (qa < f.Lq)
          atomicAdd(reinterpret_cast<float2*>(base + ((long)qa * f.nh) * HD + c),
                    make_float2(dq[nt][0] * a.scale, dq[nt][1] * a.scale));
        if (qc < f.Lq)
          atomicAdd(reinterpret_cast<float2*>(base + ((long)qc * f.nh) * HD + c),
                    make_float2(dq[nt][2] * a.scale, dq[nt][3] * a.scale));
      }
    }
    __syncthreads();                                                 // stage st and dS^T free
  }
  cp_async_wait_group<0>();
  if (f.kblk) {
    // block-indirect keys: several entries select the same source block, so the gradients
    // are added into the fp32 source-shaped buffers
    const long rs = (long)f.nh * HD;                                 // row stride of the buffers
    const long base = (long)(b / f.kb_ng) * a.kb_lsrc * rs + (long)h * HD;
    const int ja = key_a >> 6, jb = key_b >> 6;                      // logical 64-key blocks
    auto src_row = [&](int key, int j) -> long {
      return key < f.Lk ? (long)min(max(__ldg(f.kblk + (long)b * f.kb_n + j), 0), f.kb_max) * 64 + (key & 63) : -1;
    };
    const long ra = src_row(key_a, ja), rb = src_row(key_b, jb);
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      const int c = nt * 8 + 2 * t;
      if (ra >= 0) {
        atomicAdd(reinterpret_cast<float2*>(a.dk_acc + base + ra * rs + c),
                  make_float2(dk[nt][0] * a.scale, dk[nt][1] * a.scale));
        atomicAdd(reinterpret_cast<float2*>(a.dv_acc + base + ra * rs + c), make_float2(dv[nt][0], dv[nt][1]));
      }
      if (rb >= 0) {
        atomicAdd(reinterpret_cast<float2*>(a.dk_acc + base + rb * rs + c),
                  make_float2(dk[nt][2] * a.scale, dk[nt][3] * a.scale));
        atomicAdd(reinterpret_cast<float2*>(a.dv_acc + base + rb * rs + c), make_float2(dv[nt][2], dv[nt][3]));
      }
    }
    return;
  }
  // dK (scaled) and dV, bf16, straight from the accumulators
  bf16* dkg = a.dk + b * a.sdk_b + h * a.sdk_h;
  bf16* dvg = a.dv + b * a.sdv_b + h * a.sdv_h;
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) {
    const int c = nt * 8 + 2 * t;
    if (key_a < f.Lk) {
      *reinterpret_cast<uint32_t*>(dkg + (long)key_a * a.sdk_l + c) = pack_bf16(dk[nt][0] * a.scale, dk[nt][1] * a.scale);
      *reinterpret_cast<uint32_t*>(dvg + (long)key_a * a.sdv_l + c) = pack_bf16(dv[nt][0], dv[nt][1]);
    }
    if (key_b < f.Lk) {
      *reinterpret_cast<uint32_t*>(dkg + (long)key_b * a.sdk_l + c) = pack_bf16(dk[nt][2] * a.scale, dk[nt][3] * a.scale);
      *reinterpret_cast<uint32_t*>(dvg + (long)key_b * a.sdv_l + c) = pack_bf16(dv[nt][2], dv[nt][3]);
    }
  }
}

template <int HD>
size_t fwd_smem() { return (size_t)(128 + 4 * 64) * (HD + 8) * 2; }
template <int HD>
size_t bwd_smem() { return (size_t)(2 * 128 + 4 * 64) * (HD + 8) * 2 + (size_t)128 * (64 + 8) * 2 + 4 * 64 * 4; }

template <int HD>
int fwd_launch(const AttnArgs& a, cudaStream_t st) {
  const size_t sm = fwd_smem<HD>();
  dim3 grid((a.Lq + 127) / 128, a.nh, a.B);
  if (a.kblk) {
    cudaFuncSetAttribute(attn_fwd_k<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    attn_fwd_k<HD, true><<<grid, NT, sm, st>>>(a);
  } else {
    cudaFuncSetAttribute(attn_fwd_k<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    attn_fwd_k<HD, false><<<grid, NT, sm, st>>>(a);
  }
  return (int)cudaGetLastError();
}

template <int HD>
int bwd_launch(const AttnBwdArgs& a, cudaStream_t st) {
  const long rows = (long)a.f.B * a.f.nh * a.f.Lq;
  attn_bwd_pre_k<HD><<<(unsigned)((rows * 32 + NT - 1) / NT), NT, 0, st>>>(a);
  const size_t sm = bwd_smem<HD>();
  cudaFuncSetAttribute(attn_bwd_k<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  dim3 grid((a.f.Lk + 127) / 128, a.f.nh, a.f.B);
  attn_bwd_k<HD><<<grid, NT, sm, st>>>(a);
  return (int)cudaGetLastError();
}

template <int HD>
int probsum_launch(const AttnArgs& a, float* imp, cudaStream_t st) {
  const size_t sm = (size_t)2 * (128 + 64) * (HD + 8) * 2;
  cudaFuncSetAttribute(attn_probsum_k<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  dim3 grid((a.Lq + 127) / 128, (a.Lk + 63) / 64, a.B);
  attn_probsum_k<HD><<<grid, NT, sm, st>>>(a, imp);
  return (int)cudaGetLastError();
}

}  // namespace attn
}  // namespace s0

int attn_probsum_launch(const AttnArgs& a, float* imp, int hd, cudaStream_t st) {
  if (a.Lq <= 0 || a.Lk <= 0) return 0;
  if (hd == 64) return s0::attn::probsum_launch<64>(a, imp, st);
  if (hd == 128) return s0::attn::probsum_launch<128>(a, imp, st);
  return -1;
}

int attn_fwd_launch(const AttnArgs& a, int hd, cudaStream_t st) {
  if (a.Lq <= 0 || a.Lk <= 0) return 0;
  if (hd == 64) return s0::attn::fwd_launch<64>(a, st);
  if (hd == 128) return s0::attn::fwd_launch<128>(a, st);
  return -1;
}

int attn_bwd_launch(const AttnBwdArgs& a, int hd, cudaStream_t st) {
  if (a.f.Lq <= 0 || a.f.Lk <= 0) return 0;
  if (hd == 64) return s0::attn::bwd_launch<64>(a, st);
  if (hd == 128) return s0::attn::bwd_launch<128>(a, st);
  return -1;
}
