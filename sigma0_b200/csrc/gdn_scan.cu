// Cross-chunk state scan of the chunked gated delta rule (GDN / KDA), forward and
// backward, for sm_100a.
//
// The chunkwise form of the gated delta rule (the reference's _chunkwise_gdn,
// src/base_model/models/gdn.py:449-617, and the Triton WY kernel it disables, K15)
// splits into chunk-parallel work -- decay cumsums, the unit-lower-triangular WY
// solve, the intra-chunk score matrix -- and a sequential scan over chunks that
// carries the state S [HVD, HD] of every (batch, head):
//
//   vnew_c = vc_c - kc_c S_c^T                     [C, HVD]
//   o_c    = qe_c S_c^T + In_c vnew_c              [C, HVD]
//   S_c+1  = S_c * tot_c (per key column) + vnew_c^T kd_c
//
// with qe = q * exp(G), kc = (I - L)^-1 (beta k exp(G)), vc = (I - L)^-1 (beta v),
// kd = k exp(G_end - G), In = (q k^T * exp(G_i - G_j))_{i >= j}, tot = exp(G_end).
// The chunk-parallel terms are batched tensor work; this file is the scan, which is
// otherwise a host loop of small launches per 64-token chunk.  The value rows of S
// evolve independently, so one CTA owns (batch, head, VB value rows), VB = 64 or 32
// (32 when 64-row blocks would leave most SMs idle; always 32 in the backward, whose
// stages are larger): its fp32 state slice lives in registers (8 warps), and
// everything a chunk reads that does not depend on the state -- the bf16 operand
// tiles and the fp32 vc / tot (forward) or S_c / dO / vnew / tot (backward) --
// streams through a two-stage cp.async ring, so only the products sit on the
// sequential path.  Every product runs on bf16 tensor cores (mma.m16n8k16, fp32
// accumulate).  The forward saves S_c and vnew_c; the backward walks the chunks in
// reverse with the state gradient dS in registers and writes the gradients of every
// chunk operand (per value-block partials where the product sums over value rows; the
// caller adds the partials).
#include <cuda_bf16.h>

#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace gdn {

using bf16 = __nv_bfloat16;
constexpr int C = 64, NT = 256, LC = C + 8;

template <int HD, int VB, bool BWD>
struct Cfg {
  static constexpr int LH = HD + 8, LV = VB + 8;                 // padded bf16 row strides
  static constexpr int OPS_B = (3 * C * LH + C * LC) * 2;        // qe, kc, kd, In (bf16) per stage
  static constexpr int EXTRA = BWD ? (VB * HD + 2 * C * VB + HD) * 4 : (C * VB + HD) * 4;
  static constexpr int STAGE = (OPS_B + EXTRA + 15) / 16 * 16;
  static constexpr int RG = VB / 16, CG = 8 / RG;                // [VB, HD] tile: row x column groups
  static constexpr int NS = HD / CG / 8;                         // n-tiles per warp of a [VB, HD] tile
  static constexpr int NV = VB / 16;                             // n-tiles per warp of a [C, VB] tile
  static constexpr size_t SMEM = BWD ? (size_t)2 * STAGE + (size_t)(2 * VB * LH + 3 * C * LV) * 2 + RG * HD * 4
                                     : (size_t)2 * STAGE + (size_t)(VB * LH + C * LV) * 2;
};

// one chunk's state-independent operands -> a stage: bf16 qe / kc / kd [C, HD] and In [C, C]
// (padded rows), then fp32 vc [C, VB] and tot [HD] (forward) or S_c [VB, HD], dO [C, VB],
// vnew [C, VB] and tot [HD] (backward)
template <int HD, int VB, bool BWD>
__device__ __forceinline__ void load_stage(unsigned char* st, const GdnArgs& a, long cb, int v0, int tid) {
  using K = Cfg<HD, VB, BWD>;
  constexpr int LH = K::LH, CH = HD / 8;
  bf16* ops = reinterpret_cast<bf16*>(st);
  const long cbase = cb * C;
  const bf16* src[3] = {a.qe + cbase * HD, a.kc + cbase * HD, a.kd + cbase * HD};
#pragma unroll
  for (int m = 0; m < 3; ++m)
    for (int i = tid; i < C * CH; i += NT) {
      const int r = i / CH, c = i % CH;
      cp_async16(ops + m * C * LH + r * LH + c * 8, src[m] + (long)r * HD + c * 8);
    }
  const bf16* in = a.intra + cbase * C;
  for (int i = tid; i < C * (C / 8); i += NT) {
    const int r = i / (C / 8), c = i % (C / 8);
    cp_async16(ops + 3 * C * LH + r * LC + c * 8, in + (long)r * C + c * 8);
  }
  float* f = reinterpret_cast<float*>(st + K::OPS_B);
  auto rows = [&](float* dst, const float* g, long stride, int nrows, int ncols) {   // ncols % 4 == 0
    const int c4 = ncols / 4;
    for (int i = tid; i < nrows * c4; i += NT) {
      const int r = i / c4, c = i % c4;
      cp_async16(dst + r * ncols + c * 4, g + (long)r * stride + c * 4);
    }
  };
  if (!BWD) {
    rows(f, a.vc + cbase * a.HVD + v0, a.HVD, C, VB);
    rows(f + C * VB, a.tot + cb * HD, HD, 1, HD);
  } else {
    rows(f, a.S_all + (cb * a.HVD + v0) * HD, HD, VB, HD);
    rows(f + VB * HD, a.dout + cbase * a.HVD + v0, a.HVD, C, VB);
    rows(f + VB * HD + C * VB, a.vnew + cbase * a.HVD + v0, a.HVD, C, VB);
    rows(f + VB * HD + 2 * C * VB, a.tot + cb * HD, HD, 1, HD);
  }
}

// ------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------
template <int HD, int VB>
__global__ void __launch_bounds__(NT, 1) gdn_scan_fwd_k(GdnArgs a) {
  using K = Cfg<HD, VB, false>;
  constexpr int LH = K::LH, LV = K::LV, NS = K::NS, NV = K::NV, RG = K::RG, CG = K::CG;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sS = reinterpret_cast<bf16*>(smem + 2 * K::STAGE);   // S (bf16) [VB][LH]
  bf16* sV = sS + VB * LH;                                   // vnew (bf16) [C][LV]
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int HVD = a.HVD, nc = a.nc;
  const long bh = (long)b * a.nh + h;
  const int r0 = (warp & 3) * 16, cv = (warp >> 2) * (VB / 2);          // [C, VB] tiles
  const int rs = (warp % RG) * 16, cs = (warp / RG) * (HD / CG);         // [VB, HD] state tiles
  const int v0 = vb * VB;

  if (nc > 0) load_stage<HD, VB, false>(smem, a, bh * nc, v0, tid);
  cp_async_commit();
  float S[NS][4];
  {
    const float* s0 = a.S0 ? a.S0 + (bh * HVD + v0) * HD : nullptr;
#pragma unroll
    for (int nt = 0; nt < NS; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = rs + g + 8 * hf, c = cs + nt * 8 + 2 * t;
        const float2 v = s0 ? *reinterpret_cast<const float2*>(s0 + (long)r * HD + c) : make_float2(0.f, 0.f);
        S[nt][2 * hf] = v.x;
        S[nt][2 * hf + 1] = v.y;
      }
  }
  for (int c = 0; c < nc; ++c) {
    const long cb = bh * nc + c;
    // save S_c, publish its bf16 copy
#pragma unroll
    for (int nt = 0; nt < NS; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = rs + g + 8 * hf, col = cs + nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(a.S_all + (cb * HVD + v0 + r) * HD + col) =
            make_float2(S[nt][2 * hf], S[nt][2 * hf + 1]);
        *reinterpret_cast<uint32_t*>(sS + r * LH + col) = pack_bf16(S[nt][2 * hf], S[nt][2 * hf + 1]);
      }
    if (c + 1 < nc) load_stage<HD, VB, false>(smem + ((c + 1) & 1) * K::STAGE, a, cb + 1, v0, tid);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    unsigned char* cur = smem + (c & 1) * K::STAGE;
    const bf16* sQe = reinterpret_cast<const bf16*>(cur);
    const bf16 *sKc = sQe + C * LH, *sKd = sQe + 2 * C * LH, *sIn = sQe + 3 * C * LH;
    const float* vcs = reinterpret_cast<const float*>(cur + K::OPS_B);
    const float* tots = vcs + C * VB;
    // U = kc S^T, O = qe S^T  ([C, VB] tiles)
    float U[NV][4], O[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) U[i][e] = O[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ak[4], aq[4];
      load_a(ak, sKc, LH, r0, kk * 16, lane);
      load_a(aq, sQe, LH, r0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < NV / 2; ++np) {
        uint32_t bs[4];
        load_b_nk(bs, sS, LH, cv + np * 16, kk * 16, lane);
        mma_bf16(U[2 * np], ak, bs[0], bs[1]);
        mma_bf16(U[2 * np + 1], ak, bs[2], bs[3]);
        mma_bf16(O[2 * np], aq, bs[0], bs[1]);
        mma_bf16(O[2 * np + 1], aq, bs[2], bs[3]);
      }
    }
    // vnew = vc - U: saved in fp32, staged in bf16
#pragma unroll
    for (int nt = 0; nt < NV; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = r0 + g + 8 * hf, col = cv + nt * 8 + 2 * t;
        const float2 vc = *reinterpret_cast<const float2*>(vcs + r * VB + col);
        const float x = vc.x - U[nt][2 * hf], y = vc.y - U[nt][2 * hf + 1];
        *reinterpret_cast<float2*>(a.vnew + (cb * C + r) * HVD + v0 + col) = make_float2(x, y);
        *reinterpret_cast<uint32_t*>(sV + r * LV + col) = pack_bf16(x, y);
      }
    __syncthreads();
    // O += In vnew
#pragma unroll
    for (int kk = 0; kk < C / 16; ++kk) {
      uint32_t ai[4];
      load_a(ai, sIn, LC, r0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < NV / 2; ++np) {
        uint32_t bv[4];
        load_b_kn(bv, sV, LV, cv + np * 16, kk * 16, lane);
        mma_bf16(O[2 * np], ai, bv[0], bv[1]);
        mma_bf16(O[2 * np + 1], ai, bv[2], bv[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NV; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = r0 + g + 8 * hf, col = cv + nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(a.o + (cb * C + r) * HVD + v0 + col) = make_float2(O[nt][2 * hf], O[nt][2 * hf + 1]);
      }
    // S = S * tot + vnew^T kd   ([VB, HD] tile)
#pragma unroll
    for (int nt = 0; nt < NS; ++nt) {
      const float2 tv = *reinterpret_cast<const float2*>(tots + cs + nt * 8 + 2 * t);
      S[nt][0] *= tv.x;
      S[nt][1] *= tv.y;
      S[nt][2] *= tv.x;
      S[nt][3] *= tv.y;
    }
#pragma unroll
    for (int kk = 0; kk < C / 16; ++kk) {
      uint32_t av[4];
      load_a_t(av, sV, LV, rs, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < NS / 2; ++np) {
        uint32_t bk[4];
        load_b_kn(bk, sKd, LH, cs + np * 16, kk * 16, lane);
        mma_bf16(S[2 * np], av, bk[0], bk[1]);
        mma_bf16(S[2 * np + 1], av, bk[2], bk[3]);
      }
    }
    __syncthreads();                                         // sS, sV and this stage free
  }
  cp_async_wait_group<0>();
#pragma unroll
  for (int nt = 0; nt < NS; ++nt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = rs + g + 8 * hf, col = cs + nt * 8 + 2 * t;
      *reinterpret_cast<float2*>(a.S_fin + (bh * HVD + v0 + r) * HD + col) = make_float2(S[nt][2 * hf], S[nt][2 * hf + 1]);
    }
}

// ------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void neg_frag(uint32_t* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] ^= 0x80008000u;           // negate both bf16 halves
}

template <int HD, int VB>
__global__ void __launch_bounds__(NT, 1) gdn_scan_bwd_k(GdnArgs a) {
  using K = Cfg<HD, VB, true>;
  constexpr int LH = K::LH, LV = K::LV, NS = K::NS, NV = K::NV, RG = K::RG, CG = K::CG;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sS = reinterpret_cast<bf16*>(smem + 2 * K::STAGE);   // S_c (bf16) [VB][LH]
  bf16* sG = sS + VB * LH;                                   // dS_{c+1} (bf16) [VB][LH]
  bf16* sDO = sG + VB * LH;                                  // dO (bf16) [C][LV]
  bf16* sVN = sDO + C * LV;                                  // vnew (bf16) [C][LV]
  bf16* sDV = sVN + C * LV;                                  // dvnew (bf16) [C][LV]
  float* sT = reinterpret_cast<float*>(sDV + C * LV);        // dtot partials [RG][HD]
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int HVD = a.HVD, nc = a.nc;
  const long bh = (long)b * a.nh + h;
  const int r0 = (warp & 3) * 16, cv = (warp >> 2) * (VB / 2), ci = (warp >> 2) * (C / 2);
  const int rs = (warp % RG) * 16, cs = (warp / RG) * (HD / CG);
  const int ch = (warp >> 2) * (HD / 2);                     // columns of [C, HD] tiles
  const int v0 = vb * VB;
  const long nchunks = (long)a.B * a.nh * nc;                // partial-buffer stride per value block

  if (nc > 0) load_stage<HD, VB, true>(smem + ((nc - 1) & 1) * K::STAGE, a, bh * nc + nc - 1, v0, tid);
  cp_async_commit();
  float dS[NS][4];
  {
    const float* d0 = a.dS_fin ? a.dS_fin + (bh * HVD + v0) * HD : nullptr;
#pragma unroll
    for (int nt = 0; nt < NS; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = rs + g + 8 * hf, c = cs + nt * 8 + 2 * t;
        const float2 v = d0 ? *reinterpret_cast<const float2*>(d0 + (long)r * HD + c) : make_float2(0.f, 0.f);
        dS[nt][2 * hf] = v.x;
        dS[nt][2 * hf + 1] = v.y;
      }
  }
  for (int c = nc - 1; c >= 0; --c) {
    const long cb = bh * nc + c;
    if (c > 0) load_stage<HD, VB, true>(smem + ((c - 1) & 1) * K::STAGE, a, cb - 1, v0, tid);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    unsigned char* cur = smem + (c & 1) * K::STAGE;
    const bf16* sQe = reinterpret_cast<const bf16*>(cur);
    const bf16 *sKc = sQe + C * LH, *sKd = sQe + 2 * C * LH, *sIn = sQe + 3 * C * LH;
    const float* Sc = reinterpret_cast<const float*>(cur + K::OPS_B);   // [VB][HD]
    const float* dOf = Sc + VB * HD;                                    // [C][VB]
    const float* vnf = dOf + C * VB;                                    // [C][VB]
    const float* tots = vnf + C * VB;                                   // [HD]
    // stage S_c, dS_{c+1}, dO_c, vnew_c (bf16); dtot partial from the fp32 values
    float tp[NS][2];
#pragma unroll
    for (int nt = 0; nt < NS; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = rs + g + 8 * hf, col = cs + nt * 8 + 2 * t;
        const float2 sv = *reinterpret_cast<const float2*>(Sc + r * HD + col);
        *reinterpret_cast<uint32_t*>(sS + r * LH + col) = pack_bf16(sv.x, sv.y);
        *reinterpret_cast<uint32_t*>(sG + r * LH + col) = pack_bf16(dS[nt][2 * hf], dS[nt][2 * hf + 1]);
        if (hf == 0) {
          tp[nt][0] = sv.x * dS[nt][0];
          tp[nt][1] = sv.y * dS[nt][1];
        } else {
          tp[nt][0] += sv.x * dS[nt][2];
          tp[nt][1] += sv.y * dS[nt][3];
        }
      }
    for (int i = tid; i < C * (VB / 2); i += NT) {
      const int r = i / (VB / 2), c2 = (i % (VB / 2)) * 2;
      const float2 d = *reinterpret_cast<const float2*>(dOf + r * VB + c2);
      const float2 v = *reinterpret_cast<const float2*>(vnf + r * VB + c2);
      *reinterpret_cast<uint32_t*>(sDO + r * LV + c2) = pack_bf16(d.x, d.y);
      *reinterpret_cast<uint32_t*>(sVN + r * LV + c2) = pack_bf16(v.x, v.y);
    }
    // dtot: sum the 16 rows of each warp over its lanes, then the row groups in shared memory
#pragma unroll
    for (int nt = 0; nt < NS; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float x = tp[nt][e];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        tp[nt][e] = x;
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NS; ++nt) {
        sT[(warp % RG) * HD + cs + nt * 8 + 2 * t] = tp[nt][0];
        sT[(warp % RG) * HD + cs + nt * 8 + 2 * t + 1] = tp[nt][1];
      }
    }
    __syncthreads();
    if (tid < HD) {
      float x = 0.f;
#pragma unroll
      for (int q = 0; q < RG; ++q) x += sT[q * HD + tid];
      a.dtot_p[((long)vb * nchunks + cb) * HD + tid] = x;
    }
    // dvnew = In^T dO + kd dS^T   ([C, VB])
    {
      float dv[NV][4];
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) dv[i][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t ai[4];
        load_a_t(ai, sIn, LC, r0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < NV / 2; ++np) {
          uint32_t bd[4];
          load_b_kn(bd, sDO, LV, cv + np * 16, kk * 16, lane);
          mma_bf16(dv[2 * np], ai, bd[0], bd[1]);
          mma_bf16(dv[2 * np + 1], ai, bd[2], bd[3]);
        }
      }
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t ak[4];
        load_a(ak, sKd, LH, r0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < NV / 2; ++np) {
          uint32_t bg[4];
          load_b_nk(bg, sG, LH, cv + np * 16, kk * 16, lane);
          mma_bf16(dv[2 * np], ak, bg[0], bg[1]);
          mma_bf16(dv[2 * np + 1], ak, bg[2], bg[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NV; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = r0 + g + 8 * hf, col = cv + nt * 8 + 2 * t;
          *reinterpret_cast<float2*>(a.dvc + (cb * C + r) * HVD + v0 + col) = make_float2(dv[nt][2 * hf], dv[nt][2 * hf + 1]);
          *reinterpret_cast<uint32_t*>(sDV + r * LV + col) = pack_bf16(dv[nt][2 * hf], dv[nt][2 * hf + 1]);
        }
    }
    // dIn = dO vnew^T  ([C, C], summed over this block's value rows)
    {
      float di[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) di[i][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < VB / 16; ++kk) {
        uint32_t ad[4];
        load_a(ad, sDO, LV, r0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bv[4];
          load_b_nk(bv, sVN, LV, ci + np * 16, kk * 16, lane);
          mma_bf16(di[2 * np], ad, bv[0], bv[1]);
          mma_bf16(di[2 * np + 1], ad, bv[2], bv[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = r0 + g + 8 * hf, col = ci + nt * 8 + 2 * t;
          *reinterpret_cast<float2*>(a.din_p + (((long)vb * nchunks + cb) * C + r) * C + col) =
              make_float2(di[nt][2 * hf], di[nt][2 * hf + 1]);
        }
    }
    __syncthreads();
    // [C, HD] partials: dqe = dO S_c, dkc = -dvnew S_c, dkd = vnew dS_{c+1}
    {
      const long pbase = (((long)vb * nchunks + cb) * C) * HD;
#pragma unroll 1
      for (int which = 0; which < 3; ++which) {
        const bf16* A = which == 0 ? sDO : which == 1 ? sDV : sVN;
        const bf16* Bm = which == 2 ? sG : sS;
        float* dst = (which == 0 ? a.dqe_p : which == 1 ? a.dkc_p : a.dkd_p) + pbase;
        const float sgn = which == 1 ? -1.f : 1.f;
        float acc[HD / 16][4];
#pragma unroll
        for (int i = 0; i < HD / 16; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < VB / 16; ++kk) {
          uint32_t aa[4];
          load_a(aa, A, LV, r0, kk * 16, lane);
#pragma unroll
          for (int np = 0; np < HD / 32; ++np) {
            uint32_t bb[4];
            load_b_kn(bb, Bm, LH, ch + np * 16, kk * 16, lane);
            mma_bf16(acc[2 * np], aa, bb[0], bb[1]);
            mma_bf16(acc[2 * np + 1], aa, bb[2], bb[3]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < HD / 16; ++nt)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int r = r0 + g + 8 * hf, col = ch + nt * 8 + 2 * t;
            *reinterpret_cast<float2*>(dst + (long)r * HD + col) =
                make_float2(sgn * acc[nt][2 * hf], sgn * acc[nt][2 * hf + 1]);
          }
      }
    }
    // dS_c = dS_{c+1} * tot + dO^T qe - dvnew^T kc
    {
#pragma unroll
      for (int nt = 0; nt < NS; ++nt) {
        const float2 tv = *reinterpret_cast<const float2*>(tots + cs + nt * 8 + 2 * t);
        dS[nt][0] *= tv.x;
        dS[nt][1] *= tv.y;
        dS[nt][2] *= tv.x;
        dS[nt][3] *= tv.y;
      }
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t ad[4], av[4];
        load_a_t(ad, sDO, LV, rs, kk * 16, lane);
        load_a_t(av, sDV, LV, rs, kk * 16, lane);
        neg_frag(av);
#pragma unroll
        for (int np = 0; np < NS / 2; ++np) {
          uint32_t bq[4], bk[4];
          load_b_kn(bq, sQe, LH, cs + np * 16, kk * 16, lane);
          load_b_kn(bk, sKc, LH, cs + np * 16, kk * 16, lane);
          mma_bf16(dS[2 * np], ad, bq[0], bq[1]);
          mma_bf16(dS[2 * np + 1], ad, bq[2], bq[3]);
          mma_bf16(dS[2 * np], av, bk[0], bk[1]);
          mma_bf16(dS[2 * np + 1], av, bk[2], bk[3]);
        }
      }
    }
    __syncthreads();                                         // shared tiles and this stage free
  }
  cp_async_wait_group<0>();
#pragma unroll
  for (int nt = 0; nt < NS; ++nt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = rs + g + 8 * hf, col = cs + nt * 8 + 2 * t;
      *reinterpret_cast<float2*>(a.dS0 + (bh * HVD + v0 + r) * HD + col) = make_float2(dS[nt][2 * hf], dS[nt][2 * hf + 1]);
    }
}

template <int HD, int VB, bool BWD>
int launch(const GdnArgs& a, cudaStream_t st) {
  using K = Cfg<HD, VB, BWD>;
  dim3 grid(a.HVD / VB, a.nh, a.B);
  auto* kern = BWD ? gdn_scan_bwd_k<HD, VB> : gdn_scan_fwd_k<HD, VB>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM);
  kern<<<grid, NT, K::SMEM, st>>>(a);
  return (int)cudaGetLastError();
}

}  // namespace gdn
}  // namespace s0

int gdn_scan_bwd_value_block() { return 32; }

int gdn_scan_launch(const GdnArgs& a, int hd, bool bwd, int sms, cudaStream_t st) {
  using namespace s0::gdn;
  if (a.HVD % 64 || a.B <= 0 || a.nh <= 0) return -1;
  // forward: 64-row value blocks unless that leaves most SMs idle
  const bool narrow = (long)a.B * a.nh * (a.HVD / 64) < sms;
  if (hd == 64) return bwd ? launch<64, 32, true>(a, st) : narrow ? launch<64, 32, false>(a, st) : launch<64, 64, false>(a, st);
  if (hd == 128)
    return bwd ? launch<128, 32, true>(a, st) : narrow ? launch<128, 32, false>(a, st) : launch<128, 64, false>(a, st);
  return -1;
}
