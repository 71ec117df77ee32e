// Mamba-3 SISO chunked SSD for sm_100a: forward, state recompute and backward.
//
// Replaces the reference's Pallas phase-1/chunk_state/chunk_scan kernels and its
// CUDA state-scan FFI (src/base_model/models/mamba3_pallas.py:199-419,
// src/base_model/kernels/mamba3_cuda/src/siso_state_scan.cu:133-255) with a
// design where ONE thread block owns a (batch, head) pair and walks the
// sequence chunk by chunk: the P x N recurrent state never leaves the chip
// (tensor-core accumulators in registers), there are no per-chunk state
// tensors, no N-split partials and no separate state-passing pass.  RoPE,
// biases, the trapezoidal weights, the QK diagonal, D and the silu(z) gate are
// applied in-kernel.
//
// Kernels (T = B*L tokens):
//   m3_prep_fwd   per token: RMSNorm(B), RMSNorm(C) (shared by all heads),
//                 DT = softplus(dd_dt + dt_bias), ADT = A*DT, sigmoid(trap),
//                 angle rate = pi*tanh(angle)
//   m3_ssd_fwd    per (b, h): chunked scan -> gated y; optional state/angle store
//   m3_ssd_bwd    per (b, h): reverse chunk scan -> dz, dx, per-head dB/dC/dangle
//                 partials and per-token scalar gradients
//   m3_prep_bwd   per token: head reductions, BCNorm and decay-parameter chain
//
// Fixed tile geometry: chunk CS = 64, d_state N = 128, headdim P = 64, R = 32
// rope angles.  Warps own 16-row slabs; all GEMM work is bf16 mma.m16n8k16 with
// fp32 accumulation.
#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace m3 {

constexpr int CS = 64, N = 128, P = 64, R = 32, NT = 128;
constexpr int LDN = N + 8;   // bf16 row stride for N-wide tiles (conflict-free ldmatrix)
constexpr int LDP = P + 8;   // bf16 row stride for P-wide / CS-wide tiles
constexpr int RP = R + 1;    // f32 row stride for per-row angle arrays
constexpr float PI_F = 3.14159265358979323846f;
constexpr float TWO_PI_F = 6.28318530717958647692f;

using bf16 = __nv_bfloat16;

struct Geo {
  int B, L, nh, nc;
  int ldp;        // row stride of proj / dproj (elements)
  int d_inner;
  int off_B, off_C, off_dt, off_A, off_trap, off_ang;   // column offsets inside proj
};

// ---------------------------------------------------------------------------
// prep forward: one warp per token
// ---------------------------------------------------------------------------
__global__ void m3_prep_fwd(const bf16* __restrict__ proj, Geo g, const float* __restrict__ wB,
                            const float* __restrict__ wC, const float* __restrict__ dt_bias,
                            float A_floor, float eps, bf16* __restrict__ bc, float* __restrict__ dt,
                            float* __restrict__ adt, float* __restrict__ sig,
                            float* __restrict__ rate) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  int T = g.B * g.L;
  if (warp >= T) return;
  int b = warp / g.L, t = warp % g.L;
  const bf16* row = proj + (size_t)warp * g.ldp;
  // B and C: 4 elements per lane
  float xb[4], xc[4], ssb = 0.f, ssc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xb[i] = __bfloat162float(row[g.off_B + lane * 4 + i]);
    xc[i] = __bfloat162float(row[g.off_C + lane * 4 + i]);
    ssb += xb[i] * xb[i];
    ssc += xc[i] * xc[i];
  }
  ssb = warp_sum(ssb);
  ssc = warp_sum(ssc);
  float rb = rsqrtf(ssb / N + eps), rc = rsqrtf(ssc / N + eps);
  bf16* o = bc + (size_t)warp * 2 * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int n = lane * 4 + i;
    o[n] = __float2bfloat16(xb[i] * rb * wB[n]);
    o[N + n] = __float2bfloat16(xc[i] * rc * wC[n]);
  }
  for (int h = lane; h < g.nh; h += 32) {
    float ddt = __bfloat162float(row[g.off_dt + h]);
    float dA = __bfloat162float(row[g.off_A + h]);
    float tr = __bfloat162float(row[g.off_trap + h]);
    float DT = softplusf_(ddt + dt_bias[h]);
    float A = fminf(-softplusf_(dA), -A_floor);
    size_t k = ((size_t)b * g.nh + h) * g.L + t;
    dt[k] = DT;
    adt[k] = A * DT;
    sig[k] = sigmoidf_(tr);
  }
  rate[(size_t)warp * R + lane] = tanhf(__bfloat162float(row[g.off_ang + lane])) * PI_F;
}

// ---------------------------------------------------------------------------
// shared helpers for the scan kernels
// ---------------------------------------------------------------------------
struct ScanIn {
  const bf16* proj;    // z at column h*P, x at d_inner + h*P
  const bf16* bc;      // [T, 2N]  (Bn | Cn)
  const float *dt, *adt, *sig;   // [B, nh, L]
  const float* rate;   // [T, R]
  const float *Bb, *Cb, *D;      // [nh, N], [nh, N], [nh]
};

// Issue the cp.async tile loads of one chunk.
__device__ __forceinline__ void load_chunk_tiles(const ScanIn& in, const Geo& g, int b, int h, int t0,
                                                 bf16* sB, bf16* sC, bf16* sX, bf16* sZ,
                                                 const bf16* dy, bf16* sdY, int tid) {
  // B|C rows: 2N bf16 = 32 chunks of 16B
  for (int i = tid; i < CS * 32; i += NT) {
    int r = i >> 5, ch = i & 31;
    int tt = t0 + r;
    bool ok = tt < g.L;
    const bf16* src = in.bc + ((size_t)b * g.L + (ok ? tt : 0)) * 2 * N + ch * 8;
    bf16* dst = (ch < 16) ? (sB + r * LDN + ch * 8) : (sC + r * LDN + (ch - 16) * 8);
    cp_async16(dst, src, ok ? 16 : 0);
  }
  // x, z (and dy) rows: P bf16 = 8 chunks
  for (int i = tid; i < CS * 8; i += NT) {
    int r = i >> 3, ch = i & 7;
    int tt = t0 + r;
    bool ok = tt < g.L;
    size_t rowi = (size_t)b * g.L + (ok ? tt : 0);
    const bf16* px = in.proj + rowi * g.ldp + g.d_inner + h * P + ch * 8;
    const bf16* pz = in.proj + rowi * g.ldp + h * P + ch * 8;
    cp_async16(sX + r * LDP + ch * 8, px, ok ? 16 : 0);
    cp_async16(sZ + r * LDP + ch * 8, pz, ok ? 16 : 0);
    if (dy) cp_async16(sdY + r * LDP + ch * 8, dy + rowi * g.d_inner + h * P + ch * 8, ok ? 16 : 0);
  }
  cp_async_commit();
}

__device__ __forceinline__ void load_chunk_scalars(const ScanIn& in, const Geo& g, int b, int h, int t0,
                                                   float* sDT, float* sADT, float* sSig, float* sRate,
                                                   int tid) {
  size_t base = ((size_t)b * g.nh + h) * g.L;
  for (int i = tid; i <= CS; i += NT) {
    int tt = t0 + i;
    bool ok = tt < g.L;
    sDT[i] = ok ? in.dt[base + tt] : 0.f;
    sSig[i] = ok ? in.sig[base + tt] : 0.f;
    if (i < CS) sADT[i] = ok ? in.adt[base + tt] : 0.f;
  }
  for (int i = tid; i < CS * R; i += NT) {
    int r = i / R, k = i % R;
    int tt = t0 + r;
    sRate[r * RP + k] = (tt < g.L) ? in.rate[((size_t)b * g.L + tt) * R + k] : 0.f;
  }
}

// Per-row trapezoid weights and the within-chunk inclusive cumsum of ADT.
__device__ __forceinline__ void chunk_row_scalars(const float* sDT, const float* sSig, const float* sADT,
                                                  float* sGam, float* sScl, float* sCum, int tid) {
  if (tid < CS) {
    float d0 = sDT[tid], s0_ = sSig[tid], d1 = sDT[tid + 1], s1 = sSig[tid + 1];
    float gm = d0 * s0_;
    sGam[tid] = gm;
    sScl[tid] = gm + d1 * (1.f - s1);
    float v = sADT[tid];
    int lane = tid & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    sCum[tid] = v;
  }
  __syncthreads();
  if (tid >= 32 && tid < CS) sCum[tid] += sCum[31];
  __syncthreads();
}

// Angles theta[row][r] = carry[r] + sum_{i<=row} rate[i][r]*DT[i] (mod 2pi), in sTh.
// Thread layout: r = tid%32, segment = tid/32 (16 rows each).  Leaves the new
// carry (theta of row CS-1) in sNext.
__device__ __forceinline__ void chunk_angles(const float* sRate, const float* sDT, const float* sCarry,
                                             float* sTh, float* sSeg, float* sNext, int tid) {
  int r = tid & 31, seg = tid >> 5;
  float acc = 0.f;
  for (int i = 0; i < 16; ++i) {
    int row = seg * 16 + i;
    acc += sRate[row * RP + r] * sDT[row];
    sTh[row * RP + r] = acc;
  }
  sSeg[seg * 32 + r] = acc;
  __syncthreads();
  float base = sCarry[r];
  for (int s = 0; s < seg; ++s) base += sSeg[s * 32 + r];
  for (int i = 0; i < 16; ++i) {
    int row = seg * 16 + i;
    float th = base + sTh[row * RP + r];
    th = th - TWO_PI_F * floorf(th / TWO_PI_F);
    sTh[row * RP + r] = th;
    if (row == CS - 1) sNext[r] = th;
  }
  __syncthreads();
}

// Build Q = rope(Cn + cb) into sQ and K = rope(Bn + bb) * scale into sK (may alias the
// raw tiles), plus the raw dot qkr[row] = (Cn+cb).(Bn+bb).
__device__ __forceinline__ void chunk_qk(const bf16* sCn, const bf16* sBn, bf16* sQ, bf16* sK,
                                         const float* sTh, const float* sScl, const float* sCbv,
                                         const float* sBbv, float* sQKr, int tid) {
  // raw QK dot (before any in-place rewrite): 2 threads per row
  {
    int row = tid >> 1, half = tid & 1;
    float s = 0.f;
    for (int n = half * 64; n < half * 64 + 64; n += 2) {
      float2 c = unpack_bf16(*reinterpret_cast<const uint32_t*>(sCn + row * LDN + n));
      float2 bb = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + n));
      s += (c.x + sCbv[n]) * (bb.x + sBbv[n]) + (c.y + sCbv[n + 1]) * (bb.y + sBbv[n + 1]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (half == 0) sQKr[row] = s;
  }
  __syncthreads();
  // rope pairs: thread (r, seg)
  {
    int r = tid & 31, seg = tid >> 5;
    for (int i = 0; i < 16; ++i) {
      int row = seg * 16 + i;
      float sn, cs;
      sincosf(sTh[row * RP + r], &sn, &cs);
      float2 c = unpack_bf16(*reinterpret_cast<const uint32_t*>(sCn + row * LDN + 2 * r));
      float2 bb = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + 2 * r));
      float c0 = c.x + sCbv[2 * r], c1 = c.y + sCbv[2 * r + 1];
      float b0 = bb.x + sBbv[2 * r], b1 = bb.y + sBbv[2 * r + 1];
      float sc = sScl[row];
      *reinterpret_cast<uint32_t*>(sQ + row * LDN + 2 * r) = pack_bf16(c0 * cs - c1 * sn, c0 * sn + c1 * cs);
      *reinterpret_cast<uint32_t*>(sK + row * LDN + 2 * r) =
          pack_bf16((b0 * cs - b1 * sn) * sc, (b0 * sn + b1 * cs) * sc);
    }
  }
  // pass-through dims [2R, N)
  for (int i = tid; i < CS * (N - 2 * R) / 2; i += NT) {
    int row = i / ((N - 2 * R) / 2);
    int n = 2 * R + 2 * (i % ((N - 2 * R) / 2));
    float2 c = unpack_bf16(*reinterpret_cast<const uint32_t*>(sCn + row * LDN + n));
    float2 bb = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + n));
    float sc = sScl[row];
    *reinterpret_cast<uint32_t*>(sQ + row * LDN + n) = pack_bf16(c.x + sCbv[n], c.y + sCbv[n + 1]);
    *reinterpret_cast<uint32_t*>(sK + row * LDN + n) =
        pack_bf16((bb.x + sBbv[n]) * sc, (bb.y + sBbv[n + 1]) * sc);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// forward scan
// ---------------------------------------------------------------------------
struct FwdSmem {
  static constexpr size_t bytes() {
    return sizeof(bf16) * (3 * CS * LDN + 3 * CS * LDP) +
           sizeof(float) * (2 * CS * RP + 2 * (CS + 1) + 6 * CS + 2 * N + 3 * 32 + 4 * 32);
  }
};

template <bool STORE, bool WRITE_Y>
__global__ void __launch_bounds__(NT, 2)
    m3_ssd_fwd(ScanIn in, Geo g, bf16* __restrict__ y, bf16* __restrict__ states,
               float* __restrict__ theta0) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sC = reinterpret_cast<bf16*>(smem);       // Cn -> Q (in place)
  bf16* sB = sC + CS * LDN;                       // Bn -> K (in place)
  bf16* sSt = sB + CS * LDN;                      // state [p][n] (bf16)
  bf16* sX = sSt + CS * LDN;                      // V
  bf16* sZ = sX + CS * LDP;                       // z -> y staging
  bf16* sVd = sZ + CS * LDP;                      // V * decay-to-end
  float* sRate = reinterpret_cast<float*>(sVd + CS * LDP);
  float* sTh = sRate + CS * RP;
  float* sDT = sTh + CS * RP;
  float* sSig = sDT + CS + 1;
  float* sADT = sSig + CS + 1;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sQKr = sScl + CS;
  float* sW = sQKr + CS;
  float* sCbv = sW + CS;
  float* sBbv = sCbv + N;
  float* sCarry = sBbv + N;
  float* sNext = sCarry + 32;
  float* sSeg = sNext + 32;

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int m0 = warp * 16;

  for (int i = tid; i < N; i += NT) {
    sCbv[i] = in.Cb[h * N + i];
    sBbv[i] = in.Bb[h * N + i];
  }
  if (tid < 32) sCarry[tid] = 0.f;
  for (int i = tid; i < CS * LDN; i += NT) sSt[i] = __float2bfloat16(0.f);
  const float Dh = in.D[h];

  float st[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;

  for (int c = 0; c < g.nc; ++c) {
    const int t0 = c * CS;
    load_chunk_tiles(in, g, b, h, t0, sB, sC, sX, sZ, nullptr, nullptr, tid);
    load_chunk_scalars(in, g, b, h, t0, sDT, sADT, sSig, sRate, tid);
    if (STORE) {
      // state entering this chunk (bf16) and the angle carry
      bf16* dst = states + (((size_t)b * g.nh + h) * g.nc + c) * P * N;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        int n = nt * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(dst + (m0 + gq) * N + n) = pack_bf16(st[nt][0], st[nt][1]);
        *reinterpret_cast<uint32_t*>(dst + (m0 + gq + 8) * N + n) = pack_bf16(st[nt][2], st[nt][3]);
      }
      if (tid < 32) theta0[(((size_t)b * g.nh + h) * g.nc + c) * R + tid] = sCarry[tid];
    }
    cp_async_wait_all();
    __syncthreads();
    chunk_row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
    chunk_angles(sRate, sDT, sCarry, sTh, sSeg, sNext, tid);
    chunk_qk(sC, sB, sC, sB, sTh, sScl, sCbv, sBbv, sQKr, tid);
    // decay-to-end weights and V*w
    const float cend = sCum[CS - 1];
    if (tid < CS) sW[tid] = __expf(cend - sCum[tid]);
    if (tid < 32) sCarry[tid] = sNext[tid];
    __syncthreads();
    for (int i = tid; i < CS * P / 2; i += NT) {
      int r = i / (P / 2), p = 2 * (i % (P / 2));
      float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r * LDP + p));
      float w = sW[r];
      *reinterpret_cast<uint32_t*>(sVd + r * LDP + p) = pack_bf16(v.x * w, v.y * w);
    }
    __syncthreads();

    const int r0 = m0 + gq, r1 = r0 + 8;
    const float cum0 = sCum[r0], cum1 = sCum[r1];
    if (WRITE_Y) {
      // S = Q K^T (16 x 64 per warp)
      float sacc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < N / 16; ++kk) {
        uint32_t a[4];
        load_a(a, sC, LDN, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_nk(bb, sB, LDN, np * 16, kk * 16, lane);
          mma_bf16(sacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(sacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      // strictly-lower mask with decay exp(cum_l - cum_s)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int s0c = nt * 8 + 2 * tq;
        float cs0 = sCum[s0c], cs1 = sCum[s0c + 1];
        sacc[nt][0] = (s0c < r0) ? sacc[nt][0] * __expf(cum0 - cs0) : 0.f;
        sacc[nt][1] = (s0c + 1 < r0) ? sacc[nt][1] * __expf(cum0 - cs1) : 0.f;
        sacc[nt][2] = (s0c < r1) ? sacc[nt][2] * __expf(cum1 - cs0) : 0.f;
        sacc[nt][3] = (s0c + 1 < r1) ? sacc[nt][3] * __expf(cum1 - cs1) : 0.f;
      }
      // Y_off = exp(cum_l) * Q St^T
      float yacc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) yacc[i][0] = yacc[i][1] = yacc[i][2] = yacc[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < N / 16; ++kk) {
        uint32_t a[4];
        load_a(a, sC, LDN, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_nk(bb, sSt, LDN, np * 16, kk * 16, lane);
          mma_bf16(yacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(yacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      const float e0 = __expf(cum0), e1 = __expf(cum1);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        yacc[nt][0] *= e0; yacc[nt][1] *= e0; yacc[nt][2] *= e1; yacc[nt][3] *= e1;
      }
      // Y += S V
#pragma unroll
      for (int kk = 0; kk < CS / 16; ++kk) {
        uint32_t a[4];
        acc_to_a(a, sacc[2 * kk], sacc[2 * kk + 1]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sX, LDP, np * 16, kk * 16, lane);
          mma_bf16(yacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(yacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      // epilogue: + (D + qk) V, gate by silu(z); stage in sZ (own rows)
      const float q0 = Dh + sQKr[r0] * sGam[r0], q1 = Dh + sQKr[r1] * sGam[r1];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int p = nt * 8 + 2 * tq;
        float2 v0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r0 * LDP + p));
        float2 v1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r1 * LDP + p));
        float2 z0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sZ + r0 * LDP + p));
        float2 z1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sZ + r1 * LDP + p));
        float a0 = (yacc[nt][0] + q0 * v0.x) * z0.x * sigmoidf_(z0.x);
        float a1 = (yacc[nt][1] + q0 * v0.y) * z0.y * sigmoidf_(z0.y);
        float a2 = (yacc[nt][2] + q1 * v1.x) * z1.x * sigmoidf_(z1.x);
        float a3 = (yacc[nt][3] + q1 * v1.y) * z1.y * sigmoidf_(z1.y);
        *reinterpret_cast<uint32_t*>(sZ + r0 * LDP + p) = pack_bf16(a0, a1);
        *reinterpret_cast<uint32_t*>(sZ + r1 * LDP + p) = pack_bf16(a2, a3);
      }
      __syncwarp();
      for (int i = lane; i < 16 * 8; i += 32) {
        int r = i >> 3, ch = i & 7;
        int tt = t0 + m0 + r;
        if (tt < g.L)
          *reinterpret_cast<uint4*>(y + ((size_t)b * g.L + tt) * g.d_inner + h * P + ch * 8) =
              *reinterpret_cast<const uint4*>(sZ + (m0 + r) * LDP + ch * 8);
      }
    }
    // state update: st = exp(cum_end) st + Vd^T K   (rows p in [m0, m0+16))
    const float dend = __expf(cend);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      st[i][0] *= dend; st[i][1] *= dend; st[i][2] *= dend; st[i][3] *= dend;
    }
#pragma unroll
    for (int kk = 0; kk < CS / 16; ++kk) {
      uint32_t a[4];
      load_a_t(a, sVd, LDP, m0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t bb[4];
        load_b_kn(bb, sB, LDN, np * 16, kk * 16, lane);
        mma_bf16(st[2 * np], a, bb[0], bb[1]);
        mma_bf16(st[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      int n = nt * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(sSt + (m0 + gq) * LDN + n) = pack_bf16(st[nt][0], st[nt][1]);
      *reinterpret_cast<uint32_t*>(sSt + (m0 + gq + 8) * LDN + n) = pack_bf16(st[nt][2], st[nt][3]);
    }
  }
}

// ---------------------------------------------------------------------------
// backward scan
// ---------------------------------------------------------------------------
struct BwdOut {
  bf16* dproj;          // dz / dx columns are written here
  bf16* gQ;             // [T, nh, N] grad wrt C + C_bias (per head)
  bf16* gK;             // [T, nh, N] grad wrt B + B_bias (per head)
  float* gAng;          // [T, nh, R] grad wrt raw angles (per head)
  float *dgam, *dscl, *ddt, *dadt;   // [B, nh, L]
  float *dD, *dCb, *dBb;             // [B, nh], [B, nh, N], [B, nh, N]
};

struct BwdSmem {
  static constexpr size_t bytes() {
    return sizeof(bf16) * (6 * CS * LDN + 6 * CS * LDP) +
           sizeof(float) * (3 * CS * RP + 2 * (CS + 1) + 10 * CS + 4 * N + 8 * 32 + 8);
  }
};

__global__ void __launch_bounds__(NT, 1)
    m3_ssd_bwd(ScanIn in, Geo g, const bf16* __restrict__ dy, const bf16* __restrict__ states,
               const float* __restrict__ theta0, BwdOut out) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sCn = reinterpret_cast<bf16*>(smem);
  bf16* sBn = sCn + CS * LDN;
  bf16* sQ = sBn + CS * LDN;
  bf16* sK = sQ + CS * LDN;
  bf16* sSt = sK + CS * LDN;       // state entering the chunk [p][n]
  bf16* sdSt = sSt + CS * LDN;     // grad of the state leaving the chunk [p][n]
  bf16* sX = sdSt + CS * LDN;      // V -> dV staging
  bf16* sZ = sX + CS * LDP;        // z -> dz staging
  bf16* sdY = sZ + CS * LDP;       // dy -> dY0 (pre-gate grad)
  bf16* sP = sdY + CS * LDP;       // P = masked decayed S
  bf16* sdS = sP + CS * LDP;       // dS
  bf16* sdYs = sdS + CS * LDP;     // dY0 * exp(cum_l)
  float* sRate = reinterpret_cast<float*>(sdYs + CS * LDP);
  float* sTh = sRate + CS * RP;
  float* sDth = sTh + CS * RP;
  float* sDT = sDth + CS * RP;
  float* sSig = sDT + CS + 1;
  float* sADT = sSig + CS + 1;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sQKr = sScl + CS;
  float* sW = sQKr + CS;
  float* sDqk = sW + CS;
  float* sDcum = sDqk + CS;
  float* sDscl = sDcum + CS;
  float* sDTa = sDscl + CS;
  float* sCbv = sDTa + CS;
  float* sBbv = sCbv + N;
  float* sDcb = sBbv + N;
  float* sDbb = sDcb + N;
  float* sCarry = sDbb + N;        // angle carry (theta at chunk start)
  float* sNext = sCarry + 32;
  float* sSeg = sNext + 32;        // [4][32]
  float* sGc = sSeg + 4 * 32;      // reverse angle-gradient carry [32]
  float* sGseg = sGc + 32;         // [4][32] reuse region is distinct
  float* sMisc = sGseg + 32;       // [8]

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int m0 = warp * 16;
  const size_t bh = (size_t)b * g.nh + h;

  for (int i = tid; i < N; i += NT) {
    sCbv[i] = in.Cb[h * N + i];
    sBbv[i] = in.Bb[h * N + i];
    sDcb[i] = 0.f;
    sDbb[i] = 0.f;
  }
  if (tid < 32) sGc[tid] = 0.f;
  if (tid < 8) sMisc[tid] = 0.f;
  const float Dh = in.D[h];
  float dD_acc = 0.f;
  float dend_carry = 0.f;   // sum(dSout * Sout) for the chunk processed next

  float dst[16][4];   // grad of the state leaving the current chunk, rows p in [m0, m0+16)
#pragma unroll
  for (int i = 0; i < 16; ++i) dst[i][0] = dst[i][1] = dst[i][2] = dst[i][3] = 0.f;

  for (int c = g.nc - 1; c >= 0; --c) {
    const int t0 = c * CS;
    load_chunk_tiles(in, g, b, h, t0, sBn, sCn, sX, sZ, dy, sdY, tid);
    load_chunk_scalars(in, g, b, h, t0, sDT, sADT, sSig, sRate, tid);
    {
      const bf16* src = states + (bh * g.nc + c) * P * N;
      for (int i = tid; i < P * N / 8; i += NT) {
        int r = i / (N / 8), ch = i % (N / 8);
        *reinterpret_cast<uint4*>(sSt + r * LDN + ch * 8) =
            *reinterpret_cast<const uint4*>(src + r * N + ch * 8);
      }
      if (tid < 32) sCarry[tid] = theta0[(bh * g.nc + c) * R + tid];
    }
    // dSout (bf16 copy for the MMAs)
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      int n = nt * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(sdSt + (m0 + gq) * LDN + n) = pack_bf16(dst[nt][0], dst[nt][1]);
      *reinterpret_cast<uint32_t*>(sdSt + (m0 + gq + 8) * LDN + n) = pack_bf16(dst[nt][2], dst[nt][3]);
    }
    if (tid < CS) {
      sDcum[tid] = 0.f;
      sDTa[tid] = 0.f;
    }
    cp_async_wait_all();
    __syncthreads();
    chunk_row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
    chunk_angles(sRate, sDT, sCarry, sTh, sSeg, sNext, tid);
    chunk_qk(sCn, sBn, sQ, sK, sTh, sScl, sCbv, sBbv, sQKr, tid);
    const float cend = sCum[CS - 1];
    if (tid < CS) sW[tid] = __expf(cend - sCum[tid]);
    __syncthreads();

    const int r0 = m0 + gq, r1 = r0 + 8;
    const float cum0 = sCum[r0], cum1 = sCum[r1];
    const float e0 = __expf(cum0), e1 = __expf(cum1);

    // ---- recompute P and Y0; form dY0, dz -------------------------------------------------
    float pacc[8][4];   // P (fp32), rows l, cols s
    float yacc[8][4];   // Y_off -> later dY0
    float vacc[8][4];   // P V
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) pacc[i][e] = yacc[i][e] = vacc[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < N / 16; ++kk) {
      uint32_t a[4];
      load_a(a, sQ, LDN, m0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk(bb, sK, LDN, np * 16, kk * 16, lane);
        mma_bf16(pacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(pacc[2 * np + 1], a, bb[2], bb[3]);
        load_b_nk(bb, sSt, LDN, np * 16, kk * 16, lane);
        mma_bf16(yacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(yacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      int s0c = nt * 8 + 2 * tq;
      float cs0 = sCum[s0c], cs1 = sCum[s0c + 1];
      pacc[nt][0] = (s0c < r0) ? pacc[nt][0] * __expf(cum0 - cs0) : 0.f;
      pacc[nt][1] = (s0c + 1 < r0) ? pacc[nt][1] * __expf(cum0 - cs1) : 0.f;
      pacc[nt][2] = (s0c < r1) ? pacc[nt][2] * __expf(cum1 - cs0) : 0.f;
      pacc[nt][3] = (s0c + 1 < r1) ? pacc[nt][3] * __expf(cum1 - cs1) : 0.f;
      yacc[nt][0] *= e0; yacc[nt][1] *= e0; yacc[nt][2] *= e1; yacc[nt][3] *= e1;
      *reinterpret_cast<uint32_t*>(sP + r0 * LDP + s0c) = pack_bf16(pacc[nt][0], pacc[nt][1]);
      *reinterpret_cast<uint32_t*>(sP + r1 * LDP + s0c) = pack_bf16(pacc[nt][2], pacc[nt][3]);
    }
#pragma unroll
    for (int kk = 0; kk < CS / 16; ++kk) {
      uint32_t a[4];
      acc_to_a(a, pacc[2 * kk], pacc[2 * kk + 1]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_kn(bb, sX, LDP, np * 16, kk * 16, lane);
        mma_bf16(vacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(vacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    {
      const float q0 = Dh + sQKr[r0] * sGam[r0], q1 = Dh + sQKr[r1] * sGam[r1];
      float dq0 = 0.f, dq1 = 0.f, dc0 = 0.f, dc1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int p = nt * 8 + 2 * tq;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          int row = hr ? r1 : r0;
          float qd = hr ? q1 : q0;
          float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + row * LDP + p));
          float2 z = unpack_bf16(*reinterpret_cast<const uint32_t*>(sZ + row * LDP + p));
          float2 d = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY + row * LDP + p));
          float out[2];
          float vv[2] = {v.x, v.y}, zz[2] = {z.x, z.y}, dd[2] = {d.x, d.y}, dz[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            int k = hr * 2 + e;
            float yo = yacc[nt][k];
            float y0 = vacc[nt][k] + yo + qd * vv[e];
            float sg = sigmoidf_(zz[e]);
            float dy0 = dd[e] * zz[e] * sg;
            dz[e] = dd[e] * y0 * sg * (1.f + zz[e] * (1.f - sg));
            out[e] = dy0;
            yacc[nt][k] = dy0;   // keep dY0 in registers
            if (hr) { dq1 += dy0 * vv[e]; dc1 += dy0 * yo; }
            else { dq0 += dy0 * vv[e]; dc0 += dy0 * yo; }
          }
          *reinterpret_cast<uint32_t*>(sdY + row * LDP + p) = pack_bf16(out[0], out[1]);
          *reinterpret_cast<uint32_t*>(sZ + row * LDP + p) = pack_bf16(dz[0], dz[1]);
          float es = hr ? e1 : e0;
          *reinterpret_cast<uint32_t*>(sdYs + row * LDP + p) = pack_bf16(out[0] * es, out[1] * es);
        }
      }
      dq0 += __shfl_xor_sync(0xffffffffu, dq0, 1); dq0 += __shfl_xor_sync(0xffffffffu, dq0, 2);
      dq1 += __shfl_xor_sync(0xffffffffu, dq1, 1); dq1 += __shfl_xor_sync(0xffffffffu, dq1, 2);
      dc0 += __shfl_xor_sync(0xffffffffu, dc0, 1); dc0 += __shfl_xor_sync(0xffffffffu, dc0, 2);
      dc1 += __shfl_xor_sync(0xffffffffu, dc1, 1); dc1 += __shfl_xor_sync(0xffffffffu, dc1, 2);
      if (tq == 0) {
        sDqk[r0] = dq0; sDqk[r1] = dq1;
        atomicAdd(&sDcum[r0], dc0);
        atomicAdd(&sDcum[r1], dc1);
        dD_acc += dq0 + dq1;
      }
    }
    // ---- dP = dY0 V^T -> dS, G = dP*P ------------------------------------------------------
    float dsacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) dsacc[i][0] = dsacc[i][1] = dsacc[i][2] = dsacc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < P / 16; ++kk) {
      uint32_t a[4];
      acc_to_a(a, yacc[2 * kk], yacc[2 * kk + 1]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk(bb, sX, LDP, np * 16, kk * 16, lane);
        mma_bf16(dsacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(dsacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    {
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int s0c = nt * 8 + 2 * tq;
        float cs0 = sCum[s0c], cs1 = sCum[s0c + 1];
        float f00 = (s0c < r0) ? __expf(cum0 - cs0) : 0.f;
        float f01 = (s0c + 1 < r0) ? __expf(cum0 - cs1) : 0.f;
        float f10 = (s0c < r1) ? __expf(cum1 - cs0) : 0.f;
        float f11 = (s0c + 1 < r1) ? __expf(cum1 - cs1) : 0.f;
        float g00 = dsacc[nt][0] * pacc[nt][0], g01 = dsacc[nt][1] * pacc[nt][1];
        float g10 = dsacc[nt][2] * pacc[nt][2], g11 = dsacc[nt][3] * pacc[nt][3];
        rs0 += g00 + g01;
        rs1 += g10 + g11;
        float cs_a = g00 + g10, cs_b = g01 + g11;   // column partials (cols s0c, s0c+1)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          cs_a += __shfl_xor_sync(0xffffffffu, cs_a, o);
          cs_b += __shfl_xor_sync(0xffffffffu, cs_b, o);
        }
        if (gq == 0) {
          atomicAdd(&sDcum[s0c], -cs_a);
          atomicAdd(&sDcum[s0c + 1], -cs_b);
        }
        dsacc[nt][0] *= f00; dsacc[nt][1] *= f01; dsacc[nt][2] *= f10; dsacc[nt][3] *= f11;
        *reinterpret_cast<uint32_t*>(sdS + r0 * LDP + s0c) = pack_bf16(dsacc[nt][0], dsacc[nt][1]);
        *reinterpret_cast<uint32_t*>(sdS + r1 * LDP + s0c) = pack_bf16(dsacc[nt][2], dsacc[nt][3]);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1); rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1); rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      if (tq == 0) {
        atomicAdd(&sDcum[r0], rs0);
        atomicAdd(&sDcum[r1], rs1);
      }
    }
    // ---- dQ = exp(cum_l) dY0 Sin + dS K  -> gQ, dtheta, dC_bias -----------------------------
    {
      float qacc[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) qacc[i][0] = qacc[i][1] = qacc[i][2] = qacc[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < P / 16; ++kk) {
        uint32_t a[4];
        acc_to_a(a, yacc[2 * kk], yacc[2 * kk + 1]);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sSt, LDN, np * 16, kk * 16, lane);
          mma_bf16(qacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(qacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        qacc[nt][0] *= e0; qacc[nt][1] *= e0; qacc[nt][2] *= e1; qacc[nt][3] *= e1;
      }
#pragma unroll
      for (int kk = 0; kk < CS / 16; ++kk) {
        uint32_t a[4];
        acc_to_a(a, dsacc[2 * kk], dsacc[2 * kk + 1]);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sK, LDN, np * 16, kk * 16, lane);
          mma_bf16(qacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(qacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      // epilogue per element pair
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        int row = hr ? r1 : r0;
        int tt = t0 + row;
        float gm = sGam[row] * sDqk[row];
        bf16* gq_row = out.gQ + (((size_t)b * g.L + (tt < g.L ? tt : 0)) * g.nh + h) * N;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          int n = nt * 8 + 2 * tq;
          float g0 = qacc[nt][hr * 2], g1 = qacc[nt][hr * 2 + 1];
          float d0, d1;
          if (n < 2 * R) {
            int r = n >> 1;
            float sn, cs;
            sincosf(sTh[row * RP + r], &sn, &cs);
            float2 q = unpack_bf16(*reinterpret_cast<const uint32_t*>(sQ + row * LDN + n));
            sDth[row * RP + r] = -g0 * q.y + g1 * q.x;
            d0 = g0 * cs + g1 * sn;
            d1 = -g0 * sn + g1 * cs;
          } else {
            d0 = g0;
            d1 = g1;
          }
          float2 bn = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + n));
          d0 += gm * (bn.x + sBbv[n]);
          d1 += gm * (bn.y + sBbv[n + 1]);
          if (tt < g.L) *reinterpret_cast<uint32_t*>(gq_row + n) = pack_bf16(d0, d1);
          else { d0 = 0.f; d1 = 0.f; }
          qacc[nt][hr * 2] = d0;
          qacc[nt][hr * 2 + 1] = d1;
        }
      }
      // dC_bias: sum rows (2 per thread), then over gq lanes
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        float a0 = qacc[nt][0] + qacc[nt][2], a1 = qacc[nt][1] + qacc[nt][3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          a0 += __shfl_xor_sync(0xffffffffu, a0, o);
          a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        }
        if (gq == 0) {
          atomicAdd(&sDcb[nt * 8 + 2 * tq], a0);
          atomicAdd(&sDcb[nt * 8 + 2 * tq + 1], a1);
        }
      }
    }
    __syncthreads();   // sP, sdS, sdY, sdYs, sDth(Q part), sDcum complete
    // ---- dK = w_s (V dSout) + dS^T Q  -> gK, dscale, dtheta, dB_bias ------------------------
    {
      float kacc[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) kacc[i][0] = kacc[i][1] = kacc[i][2] = kacc[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < P / 16; ++kk) {
        uint32_t a[4];
        load_a(a, sX, LDP, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sdSt, LDN, np * 16, kk * 16, lane);
          mma_bf16(kacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(kacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      const float w0 = sW[r0], w1 = sW[r1];
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        kacc[nt][0] *= w0; kacc[nt][1] *= w0; kacc[nt][2] *= w1; kacc[nt][3] *= w1;
      }
#pragma unroll
      for (int kk = 0; kk < CS / 16; ++kk) {
        uint32_t a[4];
        load_a_t(a, sdS, LDP, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sQ, LDN, np * 16, kk * 16, lane);
          mma_bf16(kacc[2 * np], a, bb[0], bb[1]);
          mma_bf16(kacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      float dsc0 = 0.f, dsc1 = 0.f;
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        int row = hr ? r1 : r0;
        int tt = t0 + row;
        float sc = sScl[row];
        float gm = sGam[row] * sDqk[row];
        bf16* gk_row = out.gK + (((size_t)b * g.L + (tt < g.L ? tt : 0)) * g.nh + h) * N;
        float dsc = 0.f;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          int n = nt * 8 + 2 * tq;
          float g0 = kacc[nt][hr * 2], g1 = kacc[nt][hr * 2 + 1];
          float2 bn = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + n));
          float b0 = bn.x + sBbv[n], b1 = bn.y + sBbv[n + 1];
          float d0, d1;
          if (n < 2 * R) {
            int r = n >> 1;
            float sn, cs;
            sincosf(sTh[row * RP + r], &sn, &cs);
            float k0 = b0 * cs - b1 * sn, k1 = b0 * sn + b1 * cs;
            dsc += g0 * k0 + g1 * k1;
            float h0 = g0 * sc, h1 = g1 * sc;
            sDth[row * RP + r] += -h0 * k1 + h1 * k0;
            d0 = h0 * cs + h1 * sn;
            d1 = -h0 * sn + h1 * cs;
          } else {
            dsc += g0 * b0 + g1 * b1;
            d0 = g0 * sc;
            d1 = g1 * sc;
          }
          float2 cn = unpack_bf16(*reinterpret_cast<const uint32_t*>(sCn + row * LDN + n));
          d0 += gm * (cn.x + sCbv[n]);
          d1 += gm * (cn.y + sCbv[n + 1]);
          if (tt < g.L) *reinterpret_cast<uint32_t*>(gk_row + n) = pack_bf16(d0, d1);
          else { d0 = 0.f; d1 = 0.f; }
          kacc[nt][hr * 2] = d0;
          kacc[nt][hr * 2 + 1] = d1;
        }
        if (hr) dsc1 = dsc; else dsc0 = dsc;
      }
      dsc0 += __shfl_xor_sync(0xffffffffu, dsc0, 1); dsc0 += __shfl_xor_sync(0xffffffffu, dsc0, 2);
      dsc1 += __shfl_xor_sync(0xffffffffu, dsc1, 1); dsc1 += __shfl_xor_sync(0xffffffffu, dsc1, 2);
      if (tq == 0) { sDscl[r0] = dsc0; sDscl[r1] = dsc1; }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        float a0 = kacc[nt][0] + kacc[nt][2], a1 = kacc[nt][1] + kacc[nt][3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          a0 += __shfl_xor_sync(0xffffffffu, a0, o);
          a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        }
        if (gq == 0) {
          atomicAdd(&sDbb[nt * 8 + 2 * tq], a0);
          atomicAdd(&sDbb[nt * 8 + 2 * tq + 1], a1);
        }
      }
    }
    // ---- dV = w_s (K dSout^T) + P^T dY0 + (D+qk) dY0 -------------------------------------
    {
      float vacc2[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) vacc2[i][0] = vacc2[i][1] = vacc2[i][2] = vacc2[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < N / 16; ++kk) {
        uint32_t a[4];
        load_a(a, sK, LDN, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_nk(bb, sdSt, LDN, np * 16, kk * 16, lane);
          mma_bf16(vacc2[2 * np], a, bb[0], bb[1]);
          mma_bf16(vacc2[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      const float w0 = sW[r0], w1 = sW[r1];
      float dcs0 = 0.f, dcs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int p = nt * 8 + 2 * tq;
        float2 v0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r0 * LDP + p));
        float2 v1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r1 * LDP + p));
        vacc2[nt][0] *= w0; vacc2[nt][1] *= w0; vacc2[nt][2] *= w1; vacc2[nt][3] *= w1;
        dcs0 += v0.x * vacc2[nt][0] + v0.y * vacc2[nt][1];
        dcs1 += v1.x * vacc2[nt][2] + v1.y * vacc2[nt][3];
      }
      dcs0 += __shfl_xor_sync(0xffffffffu, dcs0, 1); dcs0 += __shfl_xor_sync(0xffffffffu, dcs0, 2);
      dcs1 += __shfl_xor_sync(0xffffffffu, dcs1, 1); dcs1 += __shfl_xor_sync(0xffffffffu, dcs1, 2);
      if (tq == 0) {
        atomicAdd(&sDcum[r0], -dcs0);
        atomicAdd(&sDcum[r1], -dcs1);
      }
#pragma unroll
      for (int kk = 0; kk < CS / 16; ++kk) {
        uint32_t a[4];
        load_a_t(a, sP, LDP, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sdY, LDP, np * 16, kk * 16, lane);
          mma_bf16(vacc2[2 * np], a, bb[0], bb[1]);
          mma_bf16(vacc2[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      const float q0 = Dh + sQKr[r0] * sGam[r0], q1 = Dh + sQKr[r1] * sGam[r1];
      __syncwarp();
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int p = nt * 8 + 2 * tq;
        float2 d0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY + r0 * LDP + p));
        float2 d1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY + r1 * LDP + p));
        *reinterpret_cast<uint32_t*>(sX + r0 * LDP + p) =
            pack_bf16(vacc2[nt][0] + q0 * d0.x, vacc2[nt][1] + q0 * d0.y);
        *reinterpret_cast<uint32_t*>(sX + r1 * LDP + p) =
            pack_bf16(vacc2[nt][2] + q1 * d1.x, vacc2[nt][3] + q1 * d1.y);
      }
      __syncwarp();
      // coalesced stores of dV (sX) and dz (sZ), own rows
      for (int i = lane; i < 16 * 8; i += 32) {
        int r = i >> 3, ch = i & 7;
        int tt = t0 + m0 + r;
        if (tt < g.L) {
          size_t rowi = ((size_t)b * g.L + tt) * g.ldp;
          *reinterpret_cast<uint4*>(out.dproj + rowi + g.d_inner + h * P + ch * 8) =
              *reinterpret_cast<const uint4*>(sX + (m0 + r) * LDP + ch * 8);
          *reinterpret_cast<uint4*>(out.dproj + rowi + h * P + ch * 8) =
              *reinterpret_cast<const uint4*>(sZ + (m0 + r) * LDP + ch * 8);
        }
      }
    }
    // ---- dSin = exp(cum_end) dSout + (dY0 e^cum)^T Q  (in place in dst) -------------------
    {
      const float dend = __expf(cend);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        dst[i][0] *= dend; dst[i][1] *= dend; dst[i][2] *= dend; dst[i][3] *= dend;
      }
#pragma unroll
      for (int kk = 0; kk < CS / 16; ++kk) {
        uint32_t a[4];
        load_a_t(a, sdYs, LDP, m0, kk * 16, lane);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bb[4];
          load_b_kn(bb, sQ, LDN, np * 16, kk * 16, lane);
          mma_bf16(dst[2 * np], a, bb[0], bb[1]);
          mma_bf16(dst[2 * np + 1], a, bb[2], bb[3]);
        }
      }
      // sum(dSin * Sin) feeds d cum_end of the previous chunk
      float dot = 0.f;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        int n = nt * 8 + 2 * tq;
        float2 s0v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sSt + (m0 + gq) * LDN + n));
        float2 s1v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sSt + (m0 + gq + 8) * LDN + n));
        dot += dst[nt][0] * s0v.x + dst[nt][1] * s0v.y + dst[nt][2] * s1v.x + dst[nt][3] * s1v.y;
      }
      dot = warp_sum(dot);
      if (lane == 0) sMisc[warp] = dot;
    }
    __syncthreads();
    // ---- per-row scalars: d cum -> dADT; angle reverse carry ------------------------------
    if (tid == 0) sDcum[CS - 1] += dend_carry;
    dend_carry = sMisc[0] + sMisc[1] + sMisc[2] + sMisc[3];
    __syncthreads();
    if (tid < CS) {
      // reverse inclusive scan of dcum: dADT[i] = sum_{t>=i} dcum[t]
      int lane2 = tid & 31;
      float v = sDcum[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        float u = __shfl_down_sync(0xffffffffu, v, o);
        if (lane2 + o < 32) v += u;
      }
      sADT[tid] = v;   // reuse as output buffer
    }
    __syncthreads();
    if (tid < 32) sADT[tid] += sADT[32];
    // angle gradient: G[row][r] = sum_{t >= row} dtheta[t][r] (global suffix sum)
    {
      int r = tid & 31, seg = tid >> 5;
      float acc = 0.f;
      for (int i = 15; i >= 0; --i) {
        int row = seg * 16 + i;
        acc += sDth[row * RP + r];
        sDth[row * RP + r] = acc;
      }
      sSeg[seg * 32 + r] = acc;
      __syncthreads();
      float base = sGc[r];
      for (int s = seg + 1; s < 4; ++s) base += sSeg[s * 32 + r];
      for (int i = 0; i < 16; ++i) {
        int row = seg * 16 + i;
        int tt = t0 + row;
        float G = base + sDth[row * RP + r];
        float rt = sRate[row * RP + r];
        float ddt_part = G * rt;
        ddt_part = warp_sum(ddt_part);   // warp == seg: all lanes share the row
        if (lane == 0) sDTa[row] = ddt_part;
        if (tt < g.L)
          out.gAng[(((size_t)b * g.L + tt) * g.nh + h) * R + r] =
              G * sDT[row] * (PI_F - rt * rt / PI_F);
        if (row == 0) sNext[r] = G;
      }
      __syncthreads();
      if (tid < 32) sGc[tid] = sNext[tid];
    }
    if (tid < CS) {
      int tt = t0 + tid;
      if (tt < g.L) {
        size_t k = bh * g.L + tt;
        out.dgam[k] = sDqk[tid] * sQKr[tid] + sDscl[tid];
        out.dscl[k] = sDscl[tid];
        out.ddt[k] = sDTa[tid];
        out.dadt[k] = sADT[tid];
      }
    }
    __syncthreads();
  }
  // per-(b,h) parameter partials
  float dd = dD_acc;
  dd = warp_sum(dd);
  if (lane == 0) sMisc[warp] = dd;
  __syncthreads();
  if (tid == 0) out.dD[bh] = sMisc[0] + sMisc[1] + sMisc[2] + sMisc[3];
  for (int i = tid; i < N; i += NT) {
    out.dCb[bh * N + i] = sDcb[i];
    out.dBb[bh * N + i] = sDbb[i];
  }
}

// ---------------------------------------------------------------------------
// prep backward: one warp per token
// ---------------------------------------------------------------------------
__global__ void m3_prep_bwd(const bf16* __restrict__ proj, Geo g, const float* __restrict__ wB,
                            const float* __restrict__ wC, const float* __restrict__ dt_bias,
                            float A_floor, float eps, const bf16* __restrict__ gQ,
                            const bf16* __restrict__ gK, const float* __restrict__ gAng,
                            const float* __restrict__ dgam, const float* __restrict__ dscl,
                            const float* __restrict__ ddt, const float* __restrict__ dadt,
                            bf16* __restrict__ dproj, float* __restrict__ dwB,
                            float* __restrict__ dwC, float* __restrict__ ddt_bias) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  int T = g.B * g.L;
  if (warp >= T) return;
  int b = warp / g.L, t = warp % g.L;
  const bf16* row = proj + (size_t)warp * g.ldp;
  bf16* drow = dproj + (size_t)warp * g.ldp;
  float sb[4] = {0, 0, 0, 0}, sc[4] = {0, 0, 0, 0}, sa = 0.f;
  for (int h = 0; h < g.nh; ++h) {
    size_t base = ((size_t)warp * g.nh + h) * N + lane * 4;
    uint2 kb = *reinterpret_cast<const uint2*>(gK + base);
    uint2 qb = *reinterpret_cast<const uint2*>(gQ + base);
    float2 k01 = unpack_bf16(kb.x), k23 = unpack_bf16(kb.y);
    float2 q01 = unpack_bf16(qb.x), q23 = unpack_bf16(qb.y);
    sb[0] += k01.x; sb[1] += k01.y; sb[2] += k23.x; sb[3] += k23.y;
    sc[0] += q01.x; sc[1] += q01.y; sc[2] += q23.x; sc[3] += q23.y;
    sa += gAng[((size_t)warp * g.nh + h) * R + lane];
  }
  // RMSNorm backward for B and C
  float xb[4], xc[4], ssb = 0.f, ssc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xb[i] = __bfloat162float(row[g.off_B + lane * 4 + i]);
    xc[i] = __bfloat162float(row[g.off_C + lane * 4 + i]);
    ssb += xb[i] * xb[i];
    ssc += xc[i] * xc[i];
  }
  ssb = warp_sum(ssb);
  ssc = warp_sum(ssc);
  float rb = rsqrtf(ssb / N + eps), rc = rsqrtf(ssc / N + eps);
  float mb = 0.f, mc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int n = lane * 4 + i;
    mb += sb[i] * wB[n] * xb[i];
    mc += sc[i] * wC[n] * xc[i];
  }
  mb = warp_sum(mb) / N;
  mc = warp_sum(mc) / N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int n = lane * 4 + i;
    float db = rb * sb[i] * wB[n] - xb[i] * rb * rb * rb * mb;
    float dc = rc * sc[i] * wC[n] - xc[i] * rc * rc * rc * mc;
    drow[g.off_B + n] = __float2bfloat16(db);
    drow[g.off_C + n] = __float2bfloat16(dc);
    atomicAdd(&dwB[n], sb[i] * xb[i] * rb);
    atomicAdd(&dwC[n], sc[i] * xc[i] * rc);
  }
  drow[g.off_ang + lane] = __float2bfloat16(sa);
  for (int h = lane; h < g.nh; h += 32) {
    float ddtr = __bfloat162float(row[g.off_dt + h]);
    float dAr = __bfloat162float(row[g.off_A + h]);
    float tr = __bfloat162float(row[g.off_trap + h]);
    float xdt = ddtr + dt_bias[h];
    float DT = softplusf_(xdt);
    float spA = softplusf_(dAr);
    float A = fminf(-spA, -A_floor);
    float sg = sigmoidf_(tr);
    size_t k = ((size_t)b * g.nh + h) * g.L + t;
    float dsp = (t > 0) ? dscl[k - 1] : 0.f;
    float dDT = ddt[k] + dgam[k] * sg + dsp * (1.f - sg) + dadt[k] * A;
    float dsg = dgam[k] * DT - dsp * DT;
    float dA = dadt[k] * DT;
    float d_ddt = dDT * sigmoidf_(xdt);
    float d_dA = (-spA < -A_floor) ? -dA * sigmoidf_(dAr) : 0.f;
    drow[g.off_dt + h] = __float2bfloat16(d_ddt);
    drow[g.off_A + h] = __float2bfloat16(d_dA);
    drow[g.off_trap + h] = __float2bfloat16(dsg * sg * (1.f - sg));
    atomicAdd(&ddt_bias[h], d_ddt);
  }
  // zero the padding columns of the row
  int used = g.off_ang + R;
  for (int c = used + lane; c < g.ldp; c += 32) drow[c] = __float2bfloat16(0.f);
}

}  // namespace m3
}  // namespace s0


// ---------------------------------------------------------------------------
// raw launchers (declared in launchers.h)
// ---------------------------------------------------------------------------
using namespace s0::m3;

static Geo make_geo(const M3Geo& G) {
  Geo g;
  g.B = G.B; g.L = G.L; g.nh = G.nh; g.nc = (G.L + CS - 1) / CS;
  g.ldp = G.ldp; g.d_inner = G.nh * P;
  g.off_B = 2 * g.d_inner; g.off_C = g.off_B + N; g.off_dt = g.off_C + N;
  g.off_A = g.off_dt + g.nh; g.off_trap = g.off_A + g.nh; g.off_ang = g.off_trap + g.nh;
  return g;
}

static ScanIn make_in(const M3Scan& S) {
  ScanIn in;
  in.proj = reinterpret_cast<const bf16*>(S.proj);
  in.bc = reinterpret_cast<const bf16*>(S.bc);
  in.dt = S.dt; in.adt = S.adt; in.sig = S.sig; in.rate = S.rate;
  in.Bb = S.Bb; in.Cb = S.Cb; in.D = S.D;
  return in;
}

int m3_nchunks(int L) { return (L + CS - 1) / CS; }

void m3_prep_fwd_launch(const M3Geo& G, const void* proj, const float* wB, const float* wC,
                        const float* dt_bias, float A_floor, float eps, void* bc, float* dt, float* adt,
                        float* sig, float* rate, cudaStream_t st) {
  Geo g = make_geo(G);
  long T = (long)g.B * g.L;
  int blocks = (int)((T * 32 + 255) / 256);
  m3_prep_fwd<<<blocks, 256, 0, st>>>(reinterpret_cast<const bf16*>(proj), g, wB, wC, dt_bias, A_floor, eps,
                                      reinterpret_cast<bf16*>(bc), dt, adt, sig, rate);
}

void m3_ssd_fwd_launch(const M3Geo& G, const M3Scan& S, void* y, void* states, float* theta0,
                       cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  size_t smem = FwdSmem::bytes();
  dim3 grid((unsigned)g.nh, (unsigned)g.B);
  bf16* yp = reinterpret_cast<bf16*>(y);
  bf16* sp = reinterpret_cast<bf16*>(states);
  if (y && states) {
    cudaFuncSetAttribute(m3_ssd_fwd<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    m3_ssd_fwd<true, true><<<grid, NT, smem, st>>>(in, g, yp, sp, theta0);
  } else if (y) {
    cudaFuncSetAttribute(m3_ssd_fwd<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    m3_ssd_fwd<false, true><<<grid, NT, smem, st>>>(in, g, yp, sp, theta0);
  } else {
    cudaFuncSetAttribute(m3_ssd_fwd<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    m3_ssd_fwd<true, false><<<grid, NT, smem, st>>>(in, g, yp, sp, theta0);
  }
}

void m3_ssd_bwd_launch(const M3Geo& G, const M3Scan& S, const void* dy, const void* states,
                       const float* theta0, const M3BwdOut& O, cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  BwdOut out;
  out.dproj = reinterpret_cast<bf16*>(O.dproj);
  out.gQ = reinterpret_cast<bf16*>(O.gQ);
  out.gK = reinterpret_cast<bf16*>(O.gK);
  out.gAng = O.gAng; out.dgam = O.dgam; out.dscl = O.dscl; out.ddt = O.ddt; out.dadt = O.dadt;
  out.dD = O.dD; out.dCb = O.dCb; out.dBb = O.dBb;
  size_t smem = BwdSmem::bytes();
  cudaFuncSetAttribute(m3_ssd_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  m3_ssd_bwd<<<dim3((unsigned)g.nh, (unsigned)g.B), NT, smem, st>>>(
      in, g, reinterpret_cast<const bf16*>(dy), reinterpret_cast<const bf16*>(states), theta0, out);
}

void m3_prep_bwd_launch(const M3Geo& G, const void* proj, const float* wB, const float* wC,
                        const float* dt_bias, float A_floor, float eps, const void* gQ, const void* gK,
                        const float* gAng, const float* dgam, const float* dscl, const float* ddt,
                        const float* dadt, void* dproj, float* dwB, float* dwC, float* ddt_bias,
                        cudaStream_t st) {
  Geo g = make_geo(G);
  long T = (long)g.B * g.L;
  int blocks = (int)((T * 32 + 255) / 256);
  m3_prep_bwd<<<blocks, 256, 0, st>>>(reinterpret_cast<const bf16*>(proj), g, wB, wC, dt_bias, A_floor, eps,
                                      reinterpret_cast<const bf16*>(gQ), reinterpret_cast<const bf16*>(gK),
                                      gAng, dgam, dscl, ddt, dadt, reinterpret_cast<bf16*>(dproj), dwB,
                                      dwC, ddt_bias);
}
