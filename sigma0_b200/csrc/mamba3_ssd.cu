// Mamba-3 SISO chunked SSD for sm_100a: forward and backward as chunk-parallel kernels.
//
// Replaces the reference's Pallas phase-1 / chunk_state / chunk_scan kernels and
// its CUDA state-scan FFI (src/base_model/models/mamba3_pallas.py:199-419,
// src/base_model/kernels/mamba3_cuda/src/siso_state_scan.cu:133-255).  RoPE,
// biases, the trapezoidal weights, the QK diagonal, D and the silu(z) gate are
// all applied inside the chunk kernels, so the only tensors between kernels are
// the per-chunk states.
//
// Every chunk kernel runs one thread block per (head, chunk, batch) -- tens of
// thousands of independent blocks -- so the tensor cores are fed by occupancy
// rather than by a sequential walk.  The cross-chunk recurrence is split into
// chunk-local work plus a cheap element-wise pass over the chunk axis:
//
//   forward:   prep -> chunk totals -> angle-carry scan -> chunk states
//              -> state passing (in place) -> chunk scan (outputs)
//   backward:  (recompute states) -> dstate contributions -> reverse state
//              passing -> chunk backward -> dtheta carry scan -> prep backward
//
// Geometry: chunk CS = 64, d_state N = 128, headdim P = 64, R = 32 rope angles.
// All matrix products are bf16 mma.m16n8k16 with fp32 accumulation.
#include "common.cuh"
#include "launchers.h"

#include <cstdlib>

namespace s0 {
namespace m3 {

constexpr int CS = 64, N = 128, P = 64, R = 32;
constexpr int LDN = N + 8;   // bf16 row stride for N-wide tiles (conflict-free ldmatrix)
constexpr int LDP = P + 8;   // bf16 row stride for 64-wide tiles
constexpr int RP = R + 4;    // f32 row stride for per-row angle arrays (16-byte rows; 4*row + r spreads banks)
constexpr float PI_F = 3.14159265358979323846f;
constexpr float TWO_PI_F = 6.28318530717958647692f;

using bf16 = __nv_bfloat16;

struct Geo {
  int B, L, nh, nc;
  int ldp;        // row stride of proj / dproj (elements)
  int d_inner;
  int off_B, off_C, off_dt, off_A, off_trap, off_ang;   // column offsets inside proj
};

struct ScanIn {
  const bf16* proj;    // z at column h*P, x at d_inner + h*P
  const bf16* bc;      // [T, 2N]  (Bn | Cn)
  const float *dt, *adt, *sig;   // [B, nh, L]
  const float* rate;   // [T, R]
  const float *Bb, *Cb, *D;      // [nh, N], [nh, N], [nh]
  const float* theta0; // [B, nh, nc, R] angle at each chunk start
  const float* aend;   // [B, nh, nc]    sum of ADT over each chunk
};


__device__ __forceinline__ float wrap2pi(float x) { return x - TWO_PI_F * floorf(x / TWO_PI_F); }

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
// chunk totals, one block per (chunk, batch) over all heads:
//   aend[h] = sum_t ADT[h][t],  angtot[h][r] = sum_t rate[t][r] * DT[h][t]
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) m3_chunk_totals(ScanIn in, Geo g, float* __restrict__ aend,
                                                       float* __restrict__ angtot) {
  __shared__ float srate[CS][R + 1];
  __shared__ float sdt[64][CS + 1];
  const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int t0 = c * CS;
  for (int i = tid; i < CS * R; i += 256) {
    int r = i / R, k = i % R;
    int tt = t0 + r;
    srate[r][k] = tt < g.L ? in.rate[((size_t)b * g.L + tt) * R + k] : 0.f;
  }
  for (int i = tid; i < g.nh * CS; i += 256) {
    int h = i / CS, r = i % CS;
    int tt = t0 + r;
    sdt[h][r] = tt < g.L ? in.dt[((size_t)b * g.nh + h) * g.L + tt] : 0.f;
  }
  __syncthreads();
  for (int o = tid; o < g.nh * R; o += 256) {
    int h = o / R, k = o % R;
    float acc = 0.f;
#pragma unroll 8
    for (int r = 0; r < CS; ++r) acc += srate[r][k] * sdt[h][r];
    angtot[((((size_t)b * g.nh + h) * g.nc) + c) * R + k] = acc;
  }
  for (int h = tid; h < g.nh; h += 256) {
    float a = 0.f;
    size_t base = ((size_t)b * g.nh + h) * g.L;
    for (int r = 0; r < CS; ++r) {
      int tt = t0 + r;
      if (tt < g.L) a += in.adt[base + tt];
    }
    aend[((size_t)b * g.nh + h) * g.nc + c] = a;
  }
}

// exclusive scan over chunks (forward, mod 2pi): theta0[c] = sum_{c'<c} angtot[c']
__global__ void m3_theta_scan(const float* __restrict__ angtot, float* __restrict__ theta0, Geo g) {
  const size_t bh = blockIdx.x;
  const int lane = threadIdx.x;
  float run = 0.f;
  constexpr int U = 8;
  for (int c0 = 0; c0 < g.nc; c0 += U) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = (c0 + u < g.nc) ? angtot[(bh * g.nc + c0 + u) * R + lane] : 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (c0 + u < g.nc) {
        theta0[(bh * g.nc + c0 + u) * R + lane] = run;
        run = wrap2pi(run + v[u]);
      }
    }
  }
}

// exclusive reverse scan over chunks, in place: x[c] = sum_{c'>c} x[c']
__global__ void m3_rev_carry(float* __restrict__ x, Geo g) {
  const size_t bh = blockIdx.x;
  const int lane = threadIdx.x;
  float run = 0.f;
  constexpr int U = 8;
  for (int k0 = 0; k0 < g.nc; k0 += U) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int c = g.nc - 1 - (k0 + u);
      v[u] = (c >= 0) ? x[(bh * g.nc + c) * R + lane] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int c = g.nc - 1 - (k0 + u);
      if (c >= 0) {
        x[(bh * g.nc + c) * R + lane] = run;
        run += v[u];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Per-chunk device helpers, templated on the block size NTH (128 or 256).
// ---------------------------------------------------------------------------
template <int NTH>
__device__ __forceinline__ void load_rows(const bf16* src_base, size_t row_stride, int col0, int ncols,
                                          bf16* dst, int ld, int t0, int L, int tid) {
  const int per = ncols / 8;
  for (int i = tid; i < CS * per; i += NTH) {
    int r = i / per, ch = i % per;
    int tt = t0 + r;
    bool ok = tt < L;
    cp_async16(dst + r * ld + ch * 8, src_base + (size_t)(ok ? tt : 0) * row_stride + col0 + ch * 8, ok ? 16 : 0);
  }
}

template <int NTH>
__device__ __forceinline__ void load_scalars(const ScanIn& in, const Geo& g, int b, int h, int t0, float* sDT,
                                             float* sADT, float* sSig, float* sRate, int tid) {
  size_t base = ((size_t)b * g.nh + h) * g.L;
  for (int i = tid; i <= CS; i += NTH) {
    int tt = t0 + i;
    bool ok = tt < g.L;
    sDT[i] = ok ? in.dt[base + tt] : 0.f;
    sSig[i] = ok ? in.sig[base + tt] : 0.f;
    if (i < CS) sADT[i] = ok ? in.adt[base + tt] : 0.f;
  }
  if (sRate) {
    for (int i = tid; i < CS * R; i += NTH) {
      int r = i / R, k = i % R;
      int tt = t0 + r;
      sRate[r * RP + k] = (tt < g.L) ? in.rate[((size_t)b * g.L + tt) * R + k] : 0.f;
    }
  }
}

// load_scalars through cp.async (zero-filled past the sequence end), so the scalar loads
// share one wait with the operand tiles instead of adding their own round trips.
template <int NTH>
__device__ __forceinline__ void load_scalars_async(const ScanIn& in, const Geo& g, int b, int h, int t0, float* sDT,
                                                   float* sADT, float* sSig, float* sRate, int tid) {
  const size_t base = ((size_t)b * g.nh + h) * g.L;
  for (int i = tid; i < 3 * (CS + 1); i += NTH) {
    const int which = i / (CS + 1), k = i % (CS + 1);
    const int tt = t0 + k;
    const bool ok = tt < g.L && (which < 2 || k < CS);
    const float* src = which == 0 ? in.dt : which == 1 ? in.sig : in.adt;
    float* dst = which == 0 ? sDT : which == 1 ? sSig : sADT;
    if (which < 2 || k < CS) cp_async4(dst + k, src + base + (ok ? tt : 0), ok ? 4 : 0);
  }
  for (int i = tid; i < CS * R; i += NTH) {
    const int r = i / R, k = i % R;
    const int tt = t0 + r;
    const bool ok = tt < g.L;
    cp_async4(sRate + r * RP + k, in.rate + ((size_t)b * g.L + (ok ? tt : 0)) * R + k, ok ? 4 : 0);
  }
}

// Group 1 of a chunk kernel's loads: scalars, rates, the head's biases (either may be
// null) and the chunk's start angle, committed as one cp.async group so the angle and
// decay prologue can start while the operand tiles (group 2) are still in flight.
template <int NTH>
__device__ __forceinline__ void load_prologue_async(const ScanIn& in, const Geo& g, int b, int h, int c, int t0,
                                                    float* sDT, float* sADT, float* sSig, float* sRate,
                                                    float* sCbv, float* sBbv, float* sTh0, int tid) {
  load_scalars_async<NTH>(in, g, b, h, t0, sDT, sADT, sSig, sRate, tid);
  const size_t bh = (size_t)b * g.nh + h;
  for (int i = tid; i < 2 * N + R; i += NTH) {   // 4-byte copies: these arrays are only 4-byte aligned
    if (i < N) { if (sCbv) cp_async4(sCbv + i, in.Cb + h * N + i); }
    else if (i < 2 * N) { if (sBbv) cp_async4(sBbv + i - N, in.Bb + h * N + i - N); }
    else cp_async4(sTh0 + i - 2 * N, in.theta0 + (bh * g.nc + c) * R + i - 2 * N);
  }
  cp_async_commit();
}

// gamma, scale and the within-chunk inclusive cumsum of ADT (needs two warps).
__device__ __forceinline__ void row_scalars(const float* sDT, const float* sSig, const float* sADT,
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

// theta[row][r] = theta0[r] + sum_{i<=row} rate[i][r] * DT[i]  (mod 2pi); writes cos/sin
// tables sCos/sSin [64][RP] (sCos doubles as the scratch for the local prefix).
template <int NTH>
__device__ __forceinline__ void chunk_angles(const float* sRate, const float* sDT, const float* th0,
                                             float* sCos, float* sSin, float* sSeg, int tid) {
  constexpr int NSEG = NTH / 32, RPS = CS / NSEG;
  int r = tid & 31, seg = tid >> 5;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    int row = seg * RPS + i;
    acc += sRate[row * RP + r] * sDT[row];
    sCos[row * RP + r] = acc;
  }
  sSeg[seg * 32 + r] = acc;
  __syncthreads();
  float base = th0[r];
  for (int s = 0; s < seg; ++s) base += sSeg[s * 32 + r];
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    int row = seg * RPS + i;
    // fast hardware sine/cosine on the angle reduced to [-pi, pi), where its absolute
    // error is ~2^-21 (far below the bf16 rounding of the rotated operands)
    const float th = base + sCos[row * RP + r];
    float sn, cs;
    __sincosf(th - TWO_PI_F * floorf(th * (1.f / TWO_PI_F) + 0.5f), &sn, &cs);
    sCos[row * RP + r] = cs;
    sSin[row * RP + r] = sn;
  }
  __syncthreads();
}

// Q = rope(Cn + cb) into sQ (may alias sCn), K = rope(Bn + bb) * scale into sK (may alias sBn);
// qkr[row] = (Cn+cb).(Bn+bb).  Either output may be skipped (nullptr; its input and bias
// pointers are then not read; qkr needs both).  Each thread owns
// 8 consecutive columns of a row (16-byte loads and stores; 16 consecutive threads share
// a row and reduce the qk dot product with shuffles); it reads its slice before writing,
// so the in-place aliasing is safe without a barrier.
template <int NTH>
__device__ __forceinline__ void build_qk(const bf16* sCn, const bf16* sBn, bf16* sQ, bf16* sK, const float* sCos,
                                         const float* sSin, const float* sScl, const float* sCbv, const float* sBbv,
                                         float* sQKr, int tid) {
  static_assert((CS * N / 8) % NTH == 0, "whole warps per iteration");
  for (int i = tid; i < CS * N / 8; i += NTH) {
    const int row = i >> 4, n0 = (i & 15) * 8;
    const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
    const float4 zf = make_float4(0.f, 0.f, 0.f, 0.f);
    const bool hq = sQ != nullptr, hk = sK != nullptr;
    const uint4 cv = hq ? *reinterpret_cast<const uint4*>(sCn + row * LDN + n0) : z4;
    const uint4 bv = hk ? *reinterpret_cast<const uint4*>(sBn + row * LDN + n0) : z4;
    const float4 cb0 = hq ? *reinterpret_cast<const float4*>(sCbv + n0) : zf;
    const float4 cb1 = hq ? *reinterpret_cast<const float4*>(sCbv + n0 + 4) : zf;
    const float4 bb0 = hk ? *reinterpret_cast<const float4*>(sBbv + n0) : zf;
    const float4 bb1 = hk ? *reinterpret_cast<const float4*>(sBbv + n0 + 4) : zf;
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
    const float cbs[8] = {cb0.x, cb0.y, cb0.z, cb0.w, cb1.x, cb1.y, cb1.z, cb1.w};
    const float bbs[8] = {bb0.x, bb0.y, bb0.z, bb0.w, bb1.x, bb1.y, bb1.z, bb1.w};
    float cq[8], bk[8];
    float qk = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 c2 = unpack_bf16(cw[k]), b2 = unpack_bf16(bw[k]);
      cq[2 * k] = c2.x + cbs[2 * k];
      cq[2 * k + 1] = c2.y + cbs[2 * k + 1];
      bk[2 * k] = b2.x + bbs[2 * k];
      bk[2 * k + 1] = b2.y + bbs[2 * k + 1];
      qk += cq[2 * k] * bk[2 * k] + cq[2 * k + 1] * bk[2 * k + 1];
    }
    if (sQKr) {
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) qk += __shfl_xor_sync(0xffffffffu, qk, o);
      if ((i & 15) == 0) sQKr[row] = qk;
    }
    if (n0 < 2 * R) {
      const float4 cs4 = *reinterpret_cast<const float4*>(sCos + row * RP + n0 / 2);
      const float4 sn4 = *reinterpret_cast<const float4*>(sSin + row * RP + n0 / 2);
      const float css[4] = {cs4.x, cs4.y, cs4.z, cs4.w}, sns[4] = {sn4.x, sn4.y, sn4.z, sn4.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float c0 = cq[2 * m], c1 = cq[2 * m + 1], b0 = bk[2 * m], b1 = bk[2 * m + 1];
        cq[2 * m] = c0 * css[m] - c1 * sns[m];
        cq[2 * m + 1] = c0 * sns[m] + c1 * css[m];
        bk[2 * m] = b0 * css[m] - b1 * sns[m];
        bk[2 * m + 1] = b0 * sns[m] + b1 * css[m];
      }
    }
    if (sQ) {
      uint4 o;
      o.x = pack_bf16(cq[0], cq[1]); o.y = pack_bf16(cq[2], cq[3]);
      o.z = pack_bf16(cq[4], cq[5]); o.w = pack_bf16(cq[6], cq[7]);
      *reinterpret_cast<uint4*>(sQ + row * LDN + n0) = o;
    }
    if (sK) {
      const float sc = sScl[row];
      uint4 o;
      o.x = pack_bf16(bk[0] * sc, bk[1] * sc); o.y = pack_bf16(bk[2] * sc, bk[3] * sc);
      o.z = pack_bf16(bk[4] * sc, bk[5] * sc); o.w = pack_bf16(bk[6] * sc, bk[7] * sc);
      *reinterpret_cast<uint4*>(sK + row * LDN + n0) = o;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ size_t state_off(const Geo& g, int b, int h, int c) {
  return ((((size_t)b * g.nh + h) * g.nc) + c) * (size_t)P * N;
}

// ---------------------------------------------------------------------------
// F3 / B2: passing along the chunk axis, in place, one element per thread.
//   forward  (REV=false): buf[c] <- S_in[c];  run = exp(aend[c]) * run + S_c[c]
//   backward (REV=true):  buf[c] <- dS_out[c]; run = exp(aend[c]) * run + U[c]
// ---------------------------------------------------------------------------
template <bool REV>
__global__ void __launch_bounds__(128) m3_pass(bf16* __restrict__ buf, const float* __restrict__ aend, Geo g,
                                              float* __restrict__ final_state) {
  const size_t bh = blockIdx.x;
  const int e8 = blockIdx.y * 128 + threadIdx.x;        // 8 consecutive elements per thread
  const size_t stride = (size_t)P * N / 8;              // in uint4 units
  uint4* base = reinterpret_cast<uint4*>(buf) + bh * g.nc * stride + e8;
  const float* ae = aend + bh * g.nc;
  float run[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) run[k] = 0.f;
  constexpr int U = 16;   // chunks in flight per thread (256 bytes): the chain is latency-bound otherwise
  for (int k0 = 0; k0 < g.nc; k0 += U) {
    uint4 v[U];
    float d[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int k = k0 + u;
      int c = REV ? g.nc - 1 - k : k;
      bool ok = k < g.nc;
      v[u] = ok ? base[(size_t)c * stride] : make_uint4(0, 0, 0, 0);
      d[u] = ok ? __expf(ae[c]) : 1.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int k = k0 + u;
      if (k < g.nc) {
        int c = REV ? g.nc - 1 - k : k;
        uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w}, o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 f = unpack_bf16(w[q]);
          o[q] = pack_bf16(run[2 * q], run[2 * q + 1]);
          run[2 * q] = d[u] * run[2 * q] + f.x;
          run[2 * q + 1] = d[u] * run[2 * q + 1] + f.y;
        }
        base[(size_t)c * stride] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  if (final_state) {   // state after the last chunk (decode prefill)
    float4* fs = reinterpret_cast<float4*>(final_state + (bh * P * N) + (size_t)e8 * 8);
    fs[0] = make_float4(run[0], run[1], run[2], run[3]);
    fs[1] = make_float4(run[4], run[5], run[6], run[7]);
  }
}

// ---------------------------------------------------------------------------
// Column-group conventions for the chunk kernels.  A block of NW warps has four
// 16-row blocks (rb = warp & 3) and CG = NW/4 column groups (cg = warp >> 2);
// 64-wide outputs give each warp 64/CG columns, 128-wide outputs 128/CG.
// ---------------------------------------------------------------------------

// F2: per-chunk state contribution S_c[p][n] = sum_s w_s V[s][p] K[s][n]   (256 threads)
constexpr size_t STATE_SMEM = sizeof(bf16) * (CS * LDN + 2 * CS * LDP) +
                              sizeof(float) * (2 * CS * RP + 2 * (CS + 4) + 5 * CS + N + 8 * 32 + 32);

__global__ void __launch_bounds__(256) m3_chunk_state(ScanIn in, Geo g, bf16* __restrict__ states) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sB = reinterpret_cast<bf16*>(smem);
  bf16* sX = sB + CS * LDN;
  bf16* sVd = sX + CS * LDP;
  float* sSin = reinterpret_cast<float*>(sVd + CS * LDP);   // rates, then sin table
  float* sCos = sSin + CS * RP;
  float* sDT = sCos + CS * RP;
  float* sSig = sDT + CS + 4;   // CS + 1 used; padded to keep later arrays 16-byte aligned
  float* sADT = sSig + CS + 4;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sW = sScl + CS;
  float* sBbv = sW + CS;
  float* sSeg = sBbv + N;
  float* sTh0 = sSeg + 8 * 32;

  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int rb = warp & 3, cg = warp >> 2;
  const int t0 = c * CS, m0 = rb * 16;
  load_prologue_async<256>(in, g, b, h, c, t0, sDT, sADT, sSig, sSin, nullptr, sBbv, sTh0, tid);
  load_rows<256>(in.bc + (size_t)b * g.L * 2 * N, 2 * N, 0, N, sB, LDN, t0, g.L, tid);
  load_rows<256>(in.proj + (size_t)b * g.L * g.ldp, g.ldp, g.d_inner + h * P, P, sX, LDP, t0, g.L, tid);
  cp_async_commit();
  cp_async_wait_group<1>();
  __syncthreads();
  row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
  chunk_angles<256>(sSin, sDT, sTh0, sCos, sSin, sSeg, tid);
  cp_async_wait_all();
  __syncthreads();
  build_qk<256>(nullptr, sB, nullptr, sB, sCos, sSin, sScl, nullptr, sBbv, nullptr, tid);
  const float cend = sCum[CS - 1];
  if (tid < CS) sW[tid] = __expf(cend - sCum[tid]);
  __syncthreads();
  for (int i = tid; i < CS * P / 2; i += 256) {
    int r = i / (P / 2), p = 2 * (i % (P / 2));
    float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + r * LDP + p));
    float w = sW[r];
    *reinterpret_cast<uint32_t*>(sVd + r * LDP + p) = pack_bf16(v.x * w, v.y * w);
  }
  __syncthreads();
  float st[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < CS / 16; ++kk) {
    uint32_t a[4];
    load_a_t(a, sVd, LDP, m0, kk * 16, lane);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bb[4];
      load_b_kn(bb, sB, LDN, cg * 64 + np * 16, kk * 16, lane);
      mma_bf16(st[2 * np], a, bb[0], bb[1]);
      mma_bf16(st[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  bf16* dst = states + state_off(g, b, h, c);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    int n = cg * 64 + nt * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(dst + (m0 + gq) * N + n) = pack_bf16(st[nt][0], st[nt][1]);
    *reinterpret_cast<uint32_t*>(dst + (m0 + gq + 8) * N + n) = pack_bf16(st[nt][2], st[nt][3]);
  }
}

// ---------------------------------------------------------------------------
// F4: chunk scan -> gated y  (256 threads: rows rb, 32-column halves cg)
// ---------------------------------------------------------------------------
constexpr size_t SCAN_SMEM = sizeof(bf16) * (3 * CS * LDN + 3 * CS * LDP) +
                             sizeof(float) * (2 * CS * RP + 2 * (CS + 4) + 5 * CS + 2 * N + 8 * 32 + 32);

__global__ void __launch_bounds__(256)
    m3_chunk_scan(ScanIn in, Geo g, const bf16* __restrict__ states, bf16* __restrict__ y) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sC = reinterpret_cast<bf16*>(smem);   // Cn -> Q
  bf16* sB = sC + CS * LDN;                   // Bn -> K
  bf16* sSt = sB + CS * LDN;                  // S_in [p][n]
  bf16* sX = sSt + CS * LDN;
  bf16* sZ = sX + CS * LDP;                   // z -> y staging
  bf16* sP = sZ + CS * LDP;
  float* sSin = reinterpret_cast<float*>(sP + CS * LDP);
  float* sCos = sSin + CS * RP;
  float* sDT = sCos + CS * RP;
  float* sSig = sDT + CS + 4;   // CS + 1 used; padded to keep later arrays 16-byte aligned
  float* sADT = sSig + CS + 4;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sQKr = sScl + CS;
  float* sCbv = sQKr + CS;
  float* sBbv = sCbv + N;
  float* sSeg = sBbv + N;
  float* sTh0 = sSeg + 8 * 32;

  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int rb = warp & 3, cg = warp >> 2, c32 = cg * 32;
  const int t0 = c * CS, m0 = rb * 16;
  const bf16* bcb = in.bc + (size_t)b * g.L * 2 * N;
  const bf16* pb = in.proj + (size_t)b * g.L * g.ldp;
  load_prologue_async<256>(in, g, b, h, c, t0, sDT, sADT, sSig, sSin, sCbv, sBbv, sTh0, tid);
  load_rows<256>(bcb, 2 * N, 0, N, sB, LDN, t0, g.L, tid);
  load_rows<256>(bcb, 2 * N, N, N, sC, LDN, t0, g.L, tid);
  load_rows<256>(pb, g.ldp, g.d_inner + h * P, P, sX, LDP, t0, g.L, tid);
  load_rows<256>(pb, g.ldp, h * P, P, sZ, LDP, t0, g.L, tid);
  {
    const bf16* src = states + state_off(g, b, h, c);
    for (int i = tid; i < P * N / 8; i += 256) {
      int r = i / (N / 8), ch = i % (N / 8);
      cp_async16(sSt + r * LDN + ch * 8, src + r * N + ch * 8);
    }
  }
  cp_async_commit();
  cp_async_wait_group<1>();
  __syncthreads();
  row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
  chunk_angles<256>(sSin, sDT, sTh0, sCos, sSin, sSeg, tid);
  cp_async_wait_all();
  __syncthreads();
  build_qk<256>(sC, sB, sC, sB, sCos, sSin, sScl, sCbv, sBbv, sQKr, tid);

  const int r0 = m0 + gq, r1 = r0 + 8;
  const float cum0 = sCum[r0], cum1 = sCum[r1];
  float sacc[4][4], yacc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) sacc[i][e] = yacc[i][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < N / 16; ++kk) {
    uint32_t a[4];
    load_a(a, sC, LDN, m0, kk * 16, lane);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t bb[4];
      load_b_nk(bb, sB, LDN, c32 + np * 16, kk * 16, lane);
      mma_bf16(sacc[2 * np], a, bb[0], bb[1]);
      mma_bf16(sacc[2 * np + 1], a, bb[2], bb[3]);
      load_b_nk(bb, sSt, LDN, c32 + np * 16, kk * 16, lane);
      mma_bf16(yacc[2 * np], a, bb[0], bb[1]);
      mma_bf16(yacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  const float e0 = __expf(cum0), e1 = __expf(cum1);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    int s0c = c32 + nt * 8 + 2 * tq;
    float cs0 = sCum[s0c], cs1 = sCum[s0c + 1];
    float p0 = (s0c < r0) ? sacc[nt][0] * __expf(cum0 - cs0) : 0.f;
    float p1 = (s0c + 1 < r0) ? sacc[nt][1] * __expf(cum0 - cs1) : 0.f;
    float p2 = (s0c < r1) ? sacc[nt][2] * __expf(cum1 - cs0) : 0.f;
    float p3 = (s0c + 1 < r1) ? sacc[nt][3] * __expf(cum1 - cs1) : 0.f;
    *reinterpret_cast<uint32_t*>(sP + r0 * LDP + s0c) = pack_bf16(p0, p1);
    *reinterpret_cast<uint32_t*>(sP + r1 * LDP + s0c) = pack_bf16(p2, p3);
    yacc[nt][0] *= e0; yacc[nt][1] *= e0; yacc[nt][2] *= e1; yacc[nt][3] *= e1;
  }
  __syncthreads();
#pragma unroll
  for (int kk = 0; kk < CS / 16; ++kk) {
    uint32_t a[4];
    load_a(a, sP, LDP, m0, kk * 16, lane);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t bb[4];
      load_b_kn(bb, sX, LDP, c32 + np * 16, kk * 16, lane);
      mma_bf16(yacc[2 * np], a, bb[0], bb[1]);
      mma_bf16(yacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  const float Dh = in.D[h];
  const float q0 = Dh + sQKr[r0] * sGam[r0], q1 = Dh + sQKr[r1] * sGam[r1];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    int p = c32 + nt * 8 + 2 * tq;
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
  __syncthreads();
  for (int i = tid; i < CS * 8; i += 256) {
    int r = i >> 3, ch = i & 7;
    int tt = t0 + r;
    if (tt < g.L)
      *reinterpret_cast<uint4*>(y + ((size_t)b * g.L + tt) * g.d_inner + h * P + ch * 8) =
          *reinterpret_cast<const uint4*>(sZ + r * LDP + ch * 8);
  }
}

// ---------------------------------------------------------------------------
// B1: per-chunk dstate contribution U_c[p][n] = sum_l exp(cum_l) dY0[l][p] Q[l][n],
// dY0 = dy * silu(z)  (256 threads: p rows rb, n halves cg)
// ---------------------------------------------------------------------------
constexpr size_t DST_SMEM = sizeof(bf16) * (CS * LDN + 2 * CS * LDP) +
                            sizeof(float) * (2 * CS * RP + 2 * (CS + 4) + 4 * CS + N + 8 * 32 + 32);

__global__ void __launch_bounds__(256)
    m3_chunk_dstate(ScanIn in, Geo g, const bf16* __restrict__ dy, bf16* __restrict__ U) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sC = reinterpret_cast<bf16*>(smem);
  bf16* sZ = sC + CS * LDN;
  bf16* sdY = sZ + CS * LDP;
  float* sSin = reinterpret_cast<float*>(sdY + CS * LDP);
  float* sCos = sSin + CS * RP;
  float* sDT = sCos + CS * RP;
  float* sSig = sDT + CS + 4;   // CS + 1 used; padded to keep later arrays 16-byte aligned
  float* sADT = sSig + CS + 4;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sCbv = sScl + CS;
  float* sSeg = sCbv + N;
  float* sTh0 = sSeg + 8 * 32;

  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int rb = warp & 3, cg = warp >> 2;
  const int t0 = c * CS, m0 = rb * 16;
  load_prologue_async<256>(in, g, b, h, c, t0, sDT, sADT, sSig, sSin, sCbv, nullptr, sTh0, tid);
  load_rows<256>(in.bc + (size_t)b * g.L * 2 * N, 2 * N, N, N, sC, LDN, t0, g.L, tid);
  load_rows<256>(in.proj + (size_t)b * g.L * g.ldp, g.ldp, h * P, P, sZ, LDP, t0, g.L, tid);
  load_rows<256>(dy + (size_t)b * g.L * g.d_inner, g.d_inner, h * P, P, sdY, LDP, t0, g.L, tid);
  cp_async_commit();
  cp_async_wait_group<1>();
  __syncthreads();
  row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
  chunk_angles<256>(sSin, sDT, sTh0, sCos, sSin, sSeg, tid);
  cp_async_wait_all();
  __syncthreads();
  build_qk<256>(sC, nullptr, sC, nullptr, sCos, sSin, sScl, sCbv, nullptr, nullptr, tid);
  for (int i = tid; i < CS * P / 2; i += 256) {
    int r = i / (P / 2), p = 2 * (i % (P / 2));
    float2 z = unpack_bf16(*reinterpret_cast<const uint32_t*>(sZ + r * LDP + p));
    float2 d = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY + r * LDP + p));
    float e = __expf(sCum[r]);
    *reinterpret_cast<uint32_t*>(sdY + r * LDP + p) =
        pack_bf16(d.x * z.x * sigmoidf_(z.x) * e, d.y * z.y * sigmoidf_(z.y) * e);
  }
  __syncthreads();
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < CS / 16; ++kk) {
    uint32_t a[4];
    load_a_t(a, sdY, LDP, m0, kk * 16, lane);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bb[4];
      load_b_kn(bb, sC, LDN, cg * 64 + np * 16, kk * 16, lane);
      mma_bf16(acc[2 * np], a, bb[0], bb[1]);
      mma_bf16(acc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  bf16* dst = U + state_off(g, b, h, c);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    int n = cg * 64 + nt * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(dst + (m0 + gq) * N + n) = pack_bf16(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<uint32_t*>(dst + (m0 + gq + 8) * N + n) = pack_bf16(acc[nt][2], acc[nt][3]);
  }
}

// ---------------------------------------------------------------------------
// B3: chunk backward (512 threads: rows rb = warp&3, column quarters cq = warp>>2)
// ---------------------------------------------------------------------------
struct BwdOut {
  bf16* dproj;          // dz / dx columns are written here
  bf16* gQ;             // [T, nh, N] grad wrt C + C_bias (per head)
  bf16* gK;             // [T, nh, N] grad wrt B + B_bias (per head)
  float* dthl;          // [T, nh, R] within-chunk suffix sums of dtheta
  float* dthtot;        // [B, nh, nc, R] chunk totals of dtheta
  float *dgam, *dscl, *dadt;         // [B, nh, L]
  float *dD, *dCb, *dBb;             // [B, nh, nc], [B, nh, nc, N] x2
};

constexpr int BWD_NT = 512;
constexpr int BPLD = 2 * N + 8;   // row stride of the bias-gradient partial-sum table (floats)
static_assert(32 * BPLD * 4 <= 2 * 64 * (N + 8) * 2, "partial table fits in the B and Q tiles");
constexpr size_t BWD_SMEM = sizeof(bf16) * (5 * CS * LDN + 6 * CS * LDP) +
                            sizeof(float) * (3 * CS * RP + 2 * (CS + 4) + 9 * CS + 4 * N + 16 * 32 + 32 + 16 +
                                             16);

__global__ void __launch_bounds__(BWD_NT, 1)
    m3_chunk_bwd(ScanIn in, Geo g, const bf16* __restrict__ dy, const bf16* __restrict__ states,
                 const bf16* __restrict__ dsout, BwdOut out) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* sBn = reinterpret_cast<bf16*>(smem);  // raw Bn
  bf16* sQ = sBn + CS * LDN;                  // Cn -> Q
  bf16* sK = sQ + CS * LDN;                   // K (rotated, scaled)
  bf16* sSt = sK + CS * LDN;                  // S_in [p][n]
  bf16* sdSt = sSt + CS * LDN;                // dS_out [p][n]
  bf16* sX = sdSt + CS * LDN;                 // V -> dV staging
  bf16* sZ = sX + CS * LDP;                   // z -> dz staging
  bf16* sdY = sZ + CS * LDP;                  // dy -> dY0
  bf16* sP = sdY + CS * LDP;
  bf16* sdS = sP + CS * LDP;
  bf16* sdY0 = sdS + CS * LDP;                // dY0 = dy * silu(z)
  float* sSin = reinterpret_cast<float*>(sdY0 + CS * LDP);
  float* sCos = sSin + CS * RP;
  float* sDth = sCos + CS * RP;
  float* sDT = sDth + CS * RP;
  float* sSig = sDT + CS + 4;   // CS + 1 used; padded to keep later arrays 16-byte aligned
  float* sADT = sSig + CS + 4;
  float* sCum = sADT + CS;
  float* sGam = sCum + CS;
  float* sScl = sGam + CS;
  float* sQKr = sScl + CS;
  float* sW = sQKr + CS;
  float* sDqk = sW + CS;
  float* sDcum = sDqk + CS;
  float* sDscl = sDcum + CS;
  float* sCbv = sDscl + CS;
  float* sBbv = sCbv + N;
  float* sSeg = sBbv + 3 * N;    // [16][32] (2N floats of spare room before it)
  float* sTh0 = sSeg + 16 * 32;  // [32]
  float* sMisc = sTh0 + 32;      // [16]
  float* sDD = sMisc + 16;       // [16]

  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const int rb = warp & 3, cq = warp >> 2;
  // 64-wide outputs: columns c16..c16+15; 128-wide outputs (dQ, dK): the 16-column
  // blocks cq and cq + 4, so every warp has one block inside the rotated half (n < 2R)
  // and one outside it and the rotation work is spread evenly
  const int c16 = cq * 16;
  const int t0 = c * CS, m0 = rb * 16;
  const size_t bh = (size_t)b * g.nh + h;
  const bf16* bcb = in.bc + (size_t)b * g.L * 2 * N;
  const bf16* pb = in.proj + (size_t)b * g.L * g.ldp;
  // group 1: the per-row scalars, rates, biases and the chunk's start angle (small);
  // group 2: the operand tiles.  The angle and decay prologue runs on group 1 while
  // group 2 is still in flight.
  load_scalars_async<BWD_NT>(in, g, b, h, t0, sDT, sADT, sSig, sSin, tid);
  for (int i = tid; i < 2 * N + R; i += BWD_NT) {   // 4-byte copies: these arrays are only 4-byte aligned
    if (i < N) cp_async4(sCbv + i, in.Cb + h * N + i);
    else if (i < 2 * N) cp_async4(sBbv + i - N, in.Bb + h * N + i - N);
    else cp_async4(sTh0 + i - 2 * N, in.theta0 + (bh * g.nc + c) * R + i - 2 * N);
  }
  cp_async_commit();
  load_rows<BWD_NT>(bcb, 2 * N, 0, N, sBn, LDN, t0, g.L, tid);
  load_rows<BWD_NT>(bcb, 2 * N, N, N, sQ, LDN, t0, g.L, tid);
  load_rows<BWD_NT>(pb, g.ldp, g.d_inner + h * P, P, sX, LDP, t0, g.L, tid);
  load_rows<BWD_NT>(pb, g.ldp, h * P, P, sZ, LDP, t0, g.L, tid);
  load_rows<BWD_NT>(dy + (size_t)b * g.L * g.d_inner, g.d_inner, h * P, P, sdY, LDP, t0, g.L, tid);
  {
    const bf16* s1 = states + state_off(g, b, h, c);
    const bf16* s2 = dsout + state_off(g, b, h, c);
    for (int i = tid; i < P * N / 8; i += BWD_NT) {
      int r = i / (N / 8), ch = i % (N / 8);
      cp_async16(sSt + r * LDN + ch * 8, s1 + r * N + ch * 8);
      cp_async16(sdSt + r * LDN + ch * 8, s2 + r * N + ch * 8);
    }
  }
  cp_async_commit();
  if (tid < CS) { sDcum[tid] = 0.f; sDscl[tid] = 0.f; }
  cp_async_wait_group<1>();
  __syncthreads();
  row_scalars(sDT, sSig, sADT, sGam, sScl, sCum, tid);
  chunk_angles<BWD_NT>(sSin, sDT, sTh0, sCos, sSin, sSeg, tid);
  cp_async_wait_all();
  __syncthreads();
  // dY0 = dy * silu(z) and the qk-diagonal row sums dqk[row] = sum_p dY0 * V (they need
  // no GEMM): one 8-column slice per thread, 8 threads per row
  for (int i = tid; i < CS * P / 8; i += BWD_NT) {
    const int row = i >> 3, p0 = (i & 7) * 8;
    const uint4 dv = *reinterpret_cast<const uint4*>(sdY + row * LDP + p0);
    const uint4 zv = *reinterpret_cast<const uint4*>(sZ + row * LDP + p0);
    const uint4 xv = *reinterpret_cast<const uint4*>(sX + row * LDP + p0);
    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t ow[4];
    float dq = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 d2 = unpack_bf16(dw[k]), z2 = unpack_bf16(zw[k]), x2 = unpack_bf16(xw[k]);
      const float a0 = d2.x * z2.x * sigmoidf_(z2.x), a1 = d2.y * z2.y * sigmoidf_(z2.y);
      dq += a0 * x2.x + a1 * x2.y;
      ow[k] = pack_bf16(a0, a1);
    }
    *reinterpret_cast<uint4*>(sdY0 + row * LDP + p0) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    dq += __shfl_xor_sync(0xffffffffu, dq, 1);
    dq += __shfl_xor_sync(0xffffffffu, dq, 2);
    dq += __shfl_xor_sync(0xffffffffu, dq, 4);
    if ((i & 7) == 0) sDqk[row] = dq;
  }
  build_qk<BWD_NT>(sQ, sBn, sQ, sK, sCos, sSin, sScl, sCbv, sBbv, sQKr, tid);
  const float cend = sCum[CS - 1];
  if (tid < CS) sW[tid] = __expf(cend - sCum[tid]);
  __syncthreads();

  const int r0 = m0 + gq, r1 = r0 + 8;
  const float cum0 = sCum[r0], cum1 = sCum[r1];
  const float e0 = __expf(cum0), e1 = __expf(cum1);
  const float Dh = in.D[h];
  const float q0 = Dh + sQKr[r0] * sGam[r0], q1 = Dh + sQKr[r1] * sGam[r1];

  // ---- A: P = masked QK^T, Y_off = Q S_in^T and dP = dY0 V^T on one (rows, cols c16..)
  // tile per warp; P and dS = dP * decay go to shared memory, G = dP * P feeds d cum --------
  float yacc[2][4];
  {
    float pacc[2][4], dsacc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) pacc[i][e] = yacc[i][e] = dsacc[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < N / 16; ++kk) {
      uint32_t a[4], bb[4];
      load_a(a, sQ, LDN, m0, kk * 16, lane);
      load_b_nk(bb, sK, LDN, c16, kk * 16, lane);
      mma_bf16(pacc[0], a, bb[0], bb[1]);
      mma_bf16(pacc[1], a, bb[2], bb[3]);
      load_b_nk(bb, sSt, LDN, c16, kk * 16, lane);
      mma_bf16(yacc[0], a, bb[0], bb[1]);
      mma_bf16(yacc[1], a, bb[2], bb[3]);
    }
#pragma unroll
    for (int kk = 0; kk < P / 16; ++kk) {
      uint32_t a[4], bb[4];
      load_a(a, sdY0, LDP, m0, kk * 16, lane);
      load_b_nk(bb, sX, LDP, c16, kk * 16, lane);
      mma_bf16(dsacc[0], a, bb[0], bb[1]);
      mma_bf16(dsacc[1], a, bb[2], bb[3]);
    }
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int s0c = c16 + nt * 8 + 2 * tq;
      const float cs0 = sCum[s0c], cs1 = sCum[s0c + 1];
      const float f00 = (s0c < r0) ? __expf(cum0 - cs0) : 0.f;
      const float f01 = (s0c + 1 < r0) ? __expf(cum0 - cs1) : 0.f;
      const float f10 = (s0c < r1) ? __expf(cum1 - cs0) : 0.f;
      const float f11 = (s0c + 1 < r1) ? __expf(cum1 - cs1) : 0.f;
      const float p00 = pacc[nt][0] * f00, p01 = pacc[nt][1] * f01;
      const float p10 = pacc[nt][2] * f10, p11 = pacc[nt][3] * f11;
      yacc[nt][0] *= e0; yacc[nt][1] *= e0; yacc[nt][2] *= e1; yacc[nt][3] *= e1;
      *reinterpret_cast<uint32_t*>(sP + r0 * LDP + s0c) = pack_bf16(p00, p01);
      *reinterpret_cast<uint32_t*>(sP + r1 * LDP + s0c) = pack_bf16(p10, p11);
      const float g00 = dsacc[nt][0] * p00, g01 = dsacc[nt][1] * p01;
      const float g10 = dsacc[nt][2] * p10, g11 = dsacc[nt][3] * p11;
      rs0 += g00 + g01;
      rs1 += g10 + g11;
      float ca = g00 + g10, cb = g01 + g11;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        ca += __shfl_xor_sync(0xffffffffu, ca, o);
        cb += __shfl_xor_sync(0xffffffffu, cb, o);
      }
      if (gq == 0) {
        atomicAdd(&sDcum[s0c], -ca);
        atomicAdd(&sDcum[s0c + 1], -cb);
      }
      *reinterpret_cast<uint32_t*>(sdS + r0 * LDP + s0c) = pack_bf16(dsacc[nt][0] * f00, dsacc[nt][1] * f01);
      *reinterpret_cast<uint32_t*>(sdS + r1 * LDP + s0c) = pack_bf16(dsacc[nt][2] * f10, dsacc[nt][3] * f11);
    }
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1); rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1); rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    if (tq == 0) {
      atomicAdd(&sDcum[r0], rs0);
      atomicAdd(&sDcum[r1], rs1);
    }
  }
  __syncthreads();   // sP, sdS complete
  // ---- B: y0 = P V + Y_off + (D + qk) V -> dz (into sZ); d cum from dY0 . Y_off ---------
  {
    float vacc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) vacc[i][0] = vacc[i][1] = vacc[i][2] = vacc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < CS / 16; ++kk) {
      uint32_t a[4], bb[4];
      load_a(a, sP, LDP, m0, kk * 16, lane);
      load_b_kn(bb, sX, LDP, c16, kk * 16, lane);
      mma_bf16(vacc[0], a, bb[0], bb[1]);
      mma_bf16(vacc[1], a, bb[2], bb[3]);
    }
    float dc0 = 0.f, dc1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int p = c16 + nt * 8 + 2 * tq;
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int row = hr ? r1 : r0;
        const float qd = hr ? q1 : q0;
        const float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(sX + row * LDP + p));
        const float2 z = unpack_bf16(*reinterpret_cast<const uint32_t*>(sZ + row * LDP + p));
        const float2 d = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY + row * LDP + p));
        const float vv[2] = {v.x, v.y}, zz[2] = {z.x, z.y}, dd[2] = {d.x, d.y};
        float dz[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = hr * 2 + e;
          const float yo = yacc[nt][k];
          const float y0 = vacc[nt][k] + yo + qd * vv[e];
          const float sg = sigmoidf_(zz[e]);
          dz[e] = dd[e] * y0 * sg * (1.f + zz[e] * (1.f - sg));
          const float dy0 = dd[e] * zz[e] * sg;
          if (hr) dc1 += dy0 * yo; else dc0 += dy0 * yo;
        }
        *reinterpret_cast<uint32_t*>(sZ + row * LDP + p) = pack_bf16(dz[0], dz[1]);
      }
    }
    dc0 += __shfl_xor_sync(0xffffffffu, dc0, 1); dc0 += __shfl_xor_sync(0xffffffffu, dc0, 2);
    dc1 += __shfl_xor_sync(0xffffffffu, dc1, 1); dc1 += __shfl_xor_sync(0xffffffffu, dc1, 2);
    if (tq == 0) {
      atomicAdd(&sDcum[r0], dc0);
      atomicAdd(&sDcum[r1], dc1);
    }
  }
  float colp[4][4];   // per-thread column partial sums of dQ / dK (bias gradients)
  // ---- C: dQ = exp(cum_l) dY0 S_in + dS K and dK = w_s (V dS_out) + dS^T Q on the same
  // columns (cq*16.. and cq*16+64..), then one epilogue for both: gQ, gK, dtheta, dscale,
  // dC_bias, dB_bias (the shared B, Q, sin/cos and bias reads happen once) ---------------
  {
    float qacc[4][4], kacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) qacc[i][e] = kacc[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < P / 16; ++kk) {
      uint32_t a[4], ax[4];
      load_a(a, sdY0, LDP, m0, kk * 16, lane);
      load_a(ax, sX, LDP, m0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bb[4];
        load_b_kn(bb, sSt, LDN, cq * 16 + np * 64, kk * 16, lane);
        mma_bf16(qacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(qacc[2 * np + 1], a, bb[2], bb[3]);
        load_b_kn(bb, sdSt, LDN, cq * 16 + np * 64, kk * 16, lane);
        mma_bf16(kacc[2 * np], ax, bb[0], bb[1]);
        mma_bf16(kacc[2 * np + 1], ax, bb[2], bb[3]);
      }
    }
    const float w0 = sW[r0], w1 = sW[r1];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      qacc[nt][0] *= e0; qacc[nt][1] *= e0; qacc[nt][2] *= e1; qacc[nt][3] *= e1;
      kacc[nt][0] *= w0; kacc[nt][1] *= w0; kacc[nt][2] *= w1; kacc[nt][3] *= w1;
    }
#pragma unroll
    for (int kk = 0; kk < CS / 16; ++kk) {
      uint32_t a[4], at[4];
      load_a(a, sdS, LDP, m0, kk * 16, lane);
      load_a_t(at, sdS, LDP, m0, kk * 16, lane);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bb[4];
        load_b_kn(bb, sK, LDN, cq * 16 + np * 64, kk * 16, lane);
        mma_bf16(qacc[2 * np], a, bb[0], bb[1]);
        mma_bf16(qacc[2 * np + 1], a, bb[2], bb[3]);
        load_b_kn(bb, sQ, LDN, cq * 16 + np * 64, kk * 16, lane);
        mma_bf16(kacc[2 * np], at, bb[0], bb[1]);
        mma_bf16(kacc[2 * np + 1], at, bb[2], bb[3]);
      }
    }
    float dsc0 = 0.f, dsc1 = 0.f;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int row = hr ? r1 : r0;
      const int tt = t0 + row;
      const bool live = tt < g.L;
      const float sc = sScl[row];
      const float gm = sGam[row] * sDqk[row];
      const size_t orow = (((size_t)b * g.L + (live ? tt : 0)) * g.nh + h) * N;
      float dsc = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int n = cq * 16 + (nt >> 1) * 64 + (nt & 1) * 8 + 2 * tq;
        const float g0 = qacc[nt][hr * 2], g1 = qacc[nt][hr * 2 + 1];
        const float k0g = kacc[nt][hr * 2], k1g = kacc[nt][hr * 2 + 1];
        const float2 bn = unpack_bf16(*reinterpret_cast<const uint32_t*>(sBn + row * LDN + n));
        const float2 bbv = *reinterpret_cast<const float2*>(sBbv + n);
        const float b0 = bn.x + bbv.x, b1 = bn.y + bbv.y;
        const float2 qv = unpack_bf16(*reinterpret_cast<const uint32_t*>(sQ + row * LDN + n));
        float dq0, dq1, dk0, dk1, cb0, cb1;
        if (nt < 2) {   // columns n < 2R: rotated
          const int r = n >> 1;
          const float sn = sSin[row * RP + r], cs = sCos[row * RP + r];
          dq0 = g0 * cs + g1 * sn;
          dq1 = -g0 * sn + g1 * cs;
          const float kr0 = b0 * cs - b1 * sn, kr1 = b0 * sn + b1 * cs;
          dsc += k0g * kr0 + k1g * kr1;
          const float h0 = k0g * sc, h1 = k1g * sc;
          sDth[row * RP + r] = (-g0 * qv.y + g1 * qv.x) + (-h0 * kr1 + h1 * kr0);
          dk0 = h0 * cs + h1 * sn;
          dk1 = -h0 * sn + h1 * cs;
          cb0 = qv.x * cs + qv.y * sn;      // C + C_bias recovered from Q (inverse rotation)
          cb1 = -qv.x * sn + qv.y * cs;
        } else {
          dq0 = g0;
          dq1 = g1;
          dsc += k0g * b0 + k1g * b1;
          dk0 = k0g * sc;
          dk1 = k1g * sc;
          cb0 = qv.x;
          cb1 = qv.y;
        }
        dq0 += gm * b0;
        dq1 += gm * b1;
        dk0 += gm * cb0;
        dk1 += gm * cb1;
        if (live) {
          *reinterpret_cast<uint32_t*>(out.gQ + orow + n) = pack_bf16(dq0, dq1);
          *reinterpret_cast<uint32_t*>(out.gK + orow + n) = pack_bf16(dk0, dk1);
        } else {
          dq0 = dq1 = dk0 = dk1 = 0.f;
        }
        qacc[nt][hr * 2] = dq0;
        qacc[nt][hr * 2 + 1] = dq1;
        kacc[nt][hr * 2] = dk0;
        kacc[nt][hr * 2 + 1] = dk1;
      }
      if (hr) dsc1 = dsc; else dsc0 = dsc;
    }
    dsc0 += __shfl_xor_sync(0xffffffffu, dsc0, 1); dsc0 += __shfl_xor_sync(0xffffffffu, dsc0, 2);
    dsc1 += __shfl_xor_sync(0xffffffffu, dsc1, 1); dsc1 += __shfl_xor_sync(0xffffffffu, dsc1, 2);
    if (tq == 0) {
      atomicAdd(&sDscl[r0], dsc0);
      atomicAdd(&sDscl[r1], dsc1);
    }
    // bias gradients: column sums over this thread's two rows; the 32 partial rows per
    // column (4 row blocks x 8 row groups) go to a table after the barrier below
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      colp[nt][0] = qacc[nt][0] + qacc[nt][2];
      colp[nt][1] = qacc[nt][1] + qacc[nt][3];
      colp[nt][2] = kacc[nt][0] + kacc[nt][2];
      colp[nt][3] = kacc[nt][1] + kacc[nt][3];
    }
  }
  __syncthreads();   // every warp done reading sX (V) as an MMA operand; sBn and sQ are dead
  {   // partial column sums -> part[32][BPLD] over the dead B and Q tiles
    float* part = reinterpret_cast<float*>(sBn);
    const int prow = rb * 8 + gq;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int n = cq * 16 + (nt >> 1) * 64 + (nt & 1) * 8 + 2 * tq;
      *reinterpret_cast<float2*>(part + prow * BPLD + n) = make_float2(colp[nt][0], colp[nt][1]);
      *reinterpret_cast<float2*>(part + prow * BPLD + N + n) = make_float2(colp[nt][2], colp[nt][3]);
    }
  }
  // the next chunk's input state (S_out of this chunk), for d cum_end after E
  uint4 nsv[P * N / 8 / BWD_NT];
  if (c + 1 < g.nc) {
    const bf16* so = states + state_off(g, b, h, c + 1);
#pragma unroll
    for (int k = 0; k < P * N / 8 / BWD_NT; ++k) {
      const int i = tid + k * BWD_NT;
      nsv[k] = *reinterpret_cast<const uint4*>(so + (i / (N / 8)) * N + (i % (N / 8)) * 8);
    }
  }
  // ---- E: dV = w_s (K dS_out^T) + P^T dY0 + (D+qk) dY0  (cols c16..) ------------------
  {
    float vacc2[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) vacc2[i][0] = vacc2[i][1] = vacc2[i][2] = vacc2[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < N / 16; ++kk) {
      uint32_t a[4], bb[4];
      load_a(a, sK, LDN, m0, kk * 16, lane);
      load_b_nk(bb, sdSt, LDN, c16, kk * 16, lane);
      mma_bf16(vacc2[0], a, bb[0], bb[1]);
      mma_bf16(vacc2[1], a, bb[2], bb[3]);
    }
    const float w0 = sW[r0], w1 = sW[r1];
    float dcs0 = 0.f, dcs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      int p = c16 + nt * 8 + 2 * tq;
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
      uint32_t a[4], bb[4];
      load_a_t(a, sP, LDP, m0, kk * 16, lane);
      load_b_kn(bb, sdY0, LDP, c16, kk * 16, lane);
      mma_bf16(vacc2[0], a, bb[0], bb[1]);
      mma_bf16(vacc2[1], a, bb[2], bb[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      int p = c16 + nt * 8 + 2 * tq;
      float2 d0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY0 + r0 * LDP + p));
      float2 d1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sdY0 + r1 * LDP + p));
      *reinterpret_cast<uint32_t*>(sX + r0 * LDP + p) =
          pack_bf16(vacc2[nt][0] + q0 * d0.x, vacc2[nt][1] + q0 * d0.y);
      *reinterpret_cast<uint32_t*>(sX + r1 * LDP + p) =
          pack_bf16(vacc2[nt][2] + q1 * d1.x, vacc2[nt][3] + q1 * d1.y);
    }
  }
  {   // d cum_end: sum(dS_out * S_out), S_out = S_in of the next chunk (no gradient past the last)
    float dot = 0.f;
    if (c + 1 < g.nc) {
#pragma unroll
      for (int kq = 0; kq < P * N / 8 / BWD_NT; ++kq) {
        const int i = tid + kq * BWD_NT;
        const int r = i / (N / 8), ch = i % (N / 8);
        const uint4 sv = nsv[kq];
        const uint4 dv = *reinterpret_cast<const uint4*>(sdSt + r * LDN + ch * 8);
        const uint32_t a[4] = {sv.x, sv.y, sv.z, sv.w}, d[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 x = unpack_bf16(a[k]), y2 = unpack_bf16(d[k]);
          dot += x.x * y2.x + x.y * y2.y;
        }
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) sMisc[warp] = dot;
  }
  // ---- F: reductions and stores ------------------------------------------------------------
  if (warp == 0) {   // dD = sum over rows of dqk (= sum_p dY0 * V)
    const float dd = warp_sum(sDqk[lane] + sDqk[lane + 32]);
    if (lane == 0) sDD[0] = dd;
  }
  __syncthreads();   // all shared atomics done; sX holds dV, sZ holds dz
  if (tid == 0) {
    float dot = 0.f, s = 0.f;
    for (int k = 0; k < BWD_NT / 32; ++k) dot += sMisc[k];
    s = sDD[0];
    sDcum[CS - 1] += dot;
    out.dD[bh * g.nc + c] = s;
  }
  for (int i = tid; i < CS * 8; i += BWD_NT) {
    int r = i >> 3, ch = i & 7;
    int tt = t0 + r;
    if (tt < g.L) {
      size_t rowi = ((size_t)b * g.L + tt) * g.ldp;
      *reinterpret_cast<uint4*>(out.dproj + rowi + g.d_inner + h * P + ch * 8) =
          *reinterpret_cast<const uint4*>(sX + r * LDP + ch * 8);
      *reinterpret_cast<uint4*>(out.dproj + rowi + h * P + ch * 8) =
          *reinterpret_cast<const uint4*>(sZ + r * LDP + ch * 8);
    }
  }
  constexpr int NSEG = BWD_NT / 32, RPS = CS / NSEG;
  {   // dtheta: within-segment suffix sums (thread r, NSEG segments of RPS rows)
    int r = tid & 31, seg = tid >> 5;
    float acc = 0.f;
#pragma unroll
    for (int i = RPS - 1; i >= 0; --i) {
      int row = seg * RPS + i;
      acc += sDth[row * RP + r];
      sDth[row * RP + r] = acc;
    }
    sSeg[seg * 32 + r] = acc;
  }
  __syncthreads();
  if (tid < CS) {   // d ADT: within-chunk reverse inclusive scan of d cum
    int l2 = tid & 31;
    float v = sDcum[tid];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float u = __shfl_down_sync(0xffffffffu, v, o);
      if (l2 + o < 32) v += u;
    }
    sADT[tid] = v;
  }
  {
    int r = tid & 31, seg = tid >> 5;
    float base = 0.f;
    for (int s = seg + 1; s < NSEG; ++s) base += sSeg[s * 32 + r];
#pragma unroll
    for (int i = 0; i < RPS; ++i) {
      int row = seg * RPS + i;
      int tt = t0 + row;
      float G = base + sDth[row * RP + r];
      if (tt < g.L) out.dthl[(((size_t)b * g.L + tt) * g.nh + h) * R + r] = G;
      if (row == 0) out.dthtot[(bh * g.nc + c) * R + r] = G;
    }
  }
  __syncthreads();
  if (tid < 32) sADT[tid] += sADT[32];
  __syncthreads();
  if (tid < CS) {
    int tt = t0 + tid;
    if (tt < g.L) {
      size_t k = bh * g.L + tt;
      out.dgam[k] = sDqk[tid] * sQKr[tid] + sDscl[tid];
      out.dscl[k] = sDscl[tid];
      out.dadt[k] = sADT[tid];
    }
  }
  {
    const float* part = reinterpret_cast<const float*>(sBn);
    for (int i = tid; i < 2 * N; i += BWD_NT) {
      float sum = 0.f;
#pragma unroll 8
      for (int r = 0; r < 32; ++r) sum += part[r * BPLD + i];
      if (i < N) out.dCb[(bh * g.nc + c) * N + i] = sum;
      else out.dBb[(bh * g.nc + c) * N + i - N] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// prep backward: warps stride over tokens; head reductions, the dtheta carry,
// BCNorm backward and the decay / trapezoid parameter chain.  The per-head angle
// term sum_r G[h][r] * rate[r] is reduced through a per-warp shared tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 2)
    m3_prep_bwd(const bf16* __restrict__ proj, Geo g, const float* __restrict__ wB,
                const float* __restrict__ wC, const float* __restrict__ dt_bias, float A_floor, float eps,
                const bf16* __restrict__ gQ, const bf16* __restrict__ gK, const float* __restrict__ dthl,
                const float* __restrict__ dthc, const float* __restrict__ dgam,
                const float* __restrict__ dscl, const float* __restrict__ dadt, bf16* __restrict__ dproj,
                float* __restrict__ dwB, float* __restrict__ dwC, float* __restrict__ ddt_bias) {
  __shared__ float tile[8][32][33];
  __shared__ float dts[8][64];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int T = g.B * g.L;
  float awB[4] = {0, 0, 0, 0}, awC[4] = {0, 0, 0, 0}, adt[2] = {0, 0};
  for (int tok = gw; tok < T; tok += nw) {
    const int b = tok / g.L, t = tok % g.L, c = t / CS;
    const bf16* row = proj + (size_t)tok * g.ldp;
    bf16* drow = dproj + (size_t)tok * g.ldp;
    for (int h = lane; h < g.nh; h += 32)
      dts[wib][h] = softplusf_(__bfloat162float(row[g.off_dt + h]) + dt_bias[h]);
    const float th = tanhf(__bfloat162float(row[g.off_ang + lane]));
    const float rt = th * PI_F;                       // angle rate (lane = r)
    const float drt = PI_F * (1.f - th * th);         // d rate / d angle
    // loads that do not depend on the head loop, issued before it so their latency
    // overlaps the head loads: the B/C row and the per-head scalars of this token
    float xb[4], xc[4];
    {
      const uint2 bv = *reinterpret_cast<const uint2*>(row + g.off_B + lane * 4);
      const uint2 cv = *reinterpret_cast<const uint2*>(row + g.off_C + lane * 4);
      const float2 b01 = unpack_bf16(bv.x), b23 = unpack_bf16(bv.y);
      const float2 c01 = unpack_bf16(cv.x), c23 = unpack_bf16(cv.y);
      xb[0] = b01.x; xb[1] = b01.y; xb[2] = b23.x; xb[3] = b23.y;
      xc[0] = c01.x; xc[1] = c01.y; xc[2] = c23.x; xc[3] = c23.y;
    }
    float hs_dgam[2], hs_dsp[2], hs_dadt[2], hs_ddtr[2], hs_dAr[2], hs_tr[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int h = lane + 32 * j;
      const bool ok = h < g.nh;
      const size_t k = ((size_t)b * g.nh + (ok ? h : 0)) * g.L + t;
      hs_dgam[j] = ok ? dgam[k] : 0.f;
      hs_dsp[j] = (ok && t > 0) ? dscl[k - 1] : 0.f;
      hs_dadt[j] = ok ? dadt[k] : 0.f;
      hs_ddtr[j] = ok ? __bfloat162float(row[g.off_dt + h]) : 0.f;
      hs_dAr[j] = ok ? __bfloat162float(row[g.off_A + h]) : 0.f;
      hs_tr[j] = ok ? __bfloat162float(row[g.off_trap + h]) : 0.f;
    }
    __syncwarp();
    float sb[4] = {0, 0, 0, 0}, sc[4] = {0, 0, 0, 0}, sa = 0.f, dang[2] = {0.f, 0.f};
    for (int h0 = 0, j = 0; h0 < g.nh; h0 += 32, ++j) {
      const int hn = min(32, g.nh - h0);
#pragma unroll 16   // 16 heads' loads in flight per warp: the head loop is latency-bound
      for (int hh = 0; hh < hn; ++hh) {
        const int h = h0 + hh;
        size_t base = ((size_t)tok * g.nh + h) * N + lane * 4;
        uint2 kb = *reinterpret_cast<const uint2*>(gK + base);
        uint2 qb = *reinterpret_cast<const uint2*>(gQ + base);
        float2 k01 = unpack_bf16(kb.x), k23 = unpack_bf16(kb.y);
        float2 q01 = unpack_bf16(qb.x), q23 = unpack_bf16(qb.y);
        sb[0] += k01.x; sb[1] += k01.y; sb[2] += k23.x; sb[3] += k23.y;
        sc[0] += q01.x; sc[1] += q01.y; sc[2] += q23.x; sc[3] += q23.y;
        float G = dthl[((size_t)tok * g.nh + h) * R + lane] +
                  dthc[(((size_t)b * g.nh + h) * g.nc + c) * R + lane];
        sa += G * dts[wib][h] * drt;
        tile[wib][hh][lane] = G * rt;
      }
      __syncwarp();
      float acc = 0.f;
      if (lane < hn) {
#pragma unroll 8
        for (int r = 0; r < R; ++r) acc += tile[wib][lane][r];
      }
      dang[j] = acc;
      __syncwarp();
    }
    float ssb = 0.f, ssc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
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
      drow[g.off_B + n] = __float2bfloat16(rb * sb[i] * wB[n] - xb[i] * rb * rb * rb * mb);
      drow[g.off_C + n] = __float2bfloat16(rc * sc[i] * wC[n] - xc[i] * rc * rc * rc * mc);
      awB[i] += sb[i] * xb[i] * rb;
      awC[i] += sc[i] * xc[i] * rc;
    }
    drow[g.off_ang + lane] = __float2bfloat16(sa);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int h = lane + 32 * j;
      if (h >= g.nh) break;
      float ddtr = hs_ddtr[j];
      float dAr = hs_dAr[j];
      float tr = hs_tr[j];
      float xdt = ddtr + dt_bias[h];
      float DT = dts[wib][h];
      float spA = softplusf_(dAr);
      float A = fminf(-spA, -A_floor);
      float sg = sigmoidf_(tr);
      float dsp = hs_dsp[j];
      float dDT = dang[j] + hs_dgam[j] * sg + dsp * (1.f - sg) + hs_dadt[j] * A;
      float dsg = hs_dgam[j] * DT - dsp * DT;
      float dA = hs_dadt[j] * DT;
      float d_ddt = dDT * sigmoidf_(xdt);
      float d_dA = (-spA < -A_floor) ? -dA * sigmoidf_(dAr) : 0.f;
      drow[g.off_dt + h] = __float2bfloat16(d_ddt);
      drow[g.off_A + h] = __float2bfloat16(d_dA);
      drow[g.off_trap + h] = __float2bfloat16(dsg * sg * (1.f - sg));
      adt[j] += d_ddt;
    }
    int used = g.off_ang + R;
    for (int cc = used + lane; cc < g.ldp; cc += 32) drow[cc] = __float2bfloat16(0.f);
    __syncwarp();
  }
  // parameter gradients: sum the 8 warps in shared memory first, then one atomic per
  // column per block (per-warp atomics all land on the same few L2 lines and serialise)
  __syncthreads();
  float* red = &tile[0][0][0];                     // [8][2N + 64]
  constexpr int RW = 2 * N + 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    red[wib * RW + lane * 4 + i] = awB[i];
    red[wib * RW + N + lane * 4 + i] = awC[i];
  }
  red[wib * RW + 2 * N + lane] = adt[0];
  red[wib * RW + 2 * N + 32 + lane] = adt[1];
  __syncthreads();
  for (int k = threadIdx.x; k < RW; k += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += red[w * RW + k];
    if (k < N) atomicAdd(&dwB[k], v);
    else if (k < 2 * N) atomicAdd(&dwC[k - N], v);
    else if (k - 2 * N < g.nh) atomicAdd(&ddt_bias[k - 2 * N], v);
  }
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
  in.theta0 = S.theta0; in.aend = S.aend;
  return in;
}

template <typename K>
static void set_smem(K kernel, size_t bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
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

void m3_chunk_totals_launch(const M3Geo& G, const M3Scan& S, float* aend, float* angtot, float* theta0,
                            cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  m3_chunk_totals<<<dim3(g.nc, g.B), 256, 0, st>>>(in, g, aend, angtot);
  m3_theta_scan<<<g.B * g.nh, 32, 0, st>>>(angtot, theta0, g);
}

void m3_states_launch(const M3Geo& G, const M3Scan& S, void* states, cudaStream_t st, float* final_state) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  set_smem(m3_chunk_state, STATE_SMEM);
  m3_chunk_state<<<dim3(g.nh, g.nc, g.B), 256, STATE_SMEM, st>>>(in, g, reinterpret_cast<bf16*>(states));
  m3_pass<false><<<dim3(g.B * g.nh, P * N / 8 / 128), 128, 0, st>>>(reinterpret_cast<bf16*>(states), S.aend, g,
                                                                          final_state);
}

void m3_scan_launch(const M3Geo& G, const M3Scan& S, const void* states, void* y, cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  set_smem(m3_chunk_scan, SCAN_SMEM);
  m3_chunk_scan<<<dim3(g.nh, g.nc, g.B), 256, SCAN_SMEM, st>>>(in, g, reinterpret_cast<const bf16*>(states),
                                                               reinterpret_cast<bf16*>(y));
}

void m3_dstates_launch(const M3Geo& G, const M3Scan& S, const void* dy, void* U, cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  set_smem(m3_chunk_dstate, DST_SMEM);
  m3_chunk_dstate<<<dim3(g.nh, g.nc, g.B), 256, DST_SMEM, st>>>(in, g, reinterpret_cast<const bf16*>(dy),
                                                                reinterpret_cast<bf16*>(U));
  m3_pass<true><<<dim3(g.B * g.nh, P * N / 8 / 128), 128, 0, st>>>(reinterpret_cast<bf16*>(U), S.aend, g, nullptr);
}

void m3_chunk_bwd_launch(const M3Geo& G, const M3Scan& S, const void* dy, const void* states, const void* dsout,
                         const M3BwdOut& O, cudaStream_t st) {
  Geo g = make_geo(G);
  ScanIn in = make_in(S);
  BwdOut out;
  out.dproj = reinterpret_cast<bf16*>(O.dproj);
  out.gQ = reinterpret_cast<bf16*>(O.gQ);
  out.gK = reinterpret_cast<bf16*>(O.gK);
  out.dthl = O.dthl; out.dthtot = O.dthtot;
  out.dgam = O.dgam; out.dscl = O.dscl; out.dadt = O.dadt;
  out.dD = O.dD; out.dCb = O.dCb; out.dBb = O.dBb;
  set_smem(m3_chunk_bwd, BWD_SMEM);
  m3_chunk_bwd<<<dim3(g.nh, g.nc, g.B), BWD_NT, BWD_SMEM, st>>>(
      in, g, reinterpret_cast<const bf16*>(dy), reinterpret_cast<const bf16*>(states),
      reinterpret_cast<const bf16*>(dsout), out);
  m3_rev_carry<<<g.B * g.nh, 32, 0, st>>>(O.dthtot, g);
}

void m3_rev_carry_launch(const M3Geo& G, float* dthtot, cudaStream_t st) {
  Geo g = make_geo(G);
  m3_rev_carry<<<g.B * g.nh, 32, 0, st>>>(dthtot, g);
}

void m3_prep_bwd_launch(const M3Geo& G, const void* proj, const float* wB, const float* wC,
                        const float* dt_bias, float A_floor, float eps, const void* gQ, const void* gK,
                        const float* dthl, const float* dthc, const float* dgam, const float* dscl,
                        const float* dadt, void* dproj, float* dwB, float* dwC, float* ddt_bias,
                        cudaStream_t st) {
  Geo g = make_geo(G);
  long T = (long)g.B * g.L;
  int blocks = (int)((T * 32 + 255) / 256);
  if (blocks > 148 * 2) blocks = 148 * 2;   // one wave at two 256-thread blocks per SM
  m3_prep_bwd<<<blocks, 256, 0, st>>>(reinterpret_cast<const bf16*>(proj), g, wB, wC, dt_bias, A_floor, eps,
                                      reinterpret_cast<const bf16*>(gQ), reinterpret_cast<const bf16*>(gK),
                                      dthl, dthc, dgam, dscl, dadt, reinterpret_cast<bf16*>(dproj), dwB, dwC,
                                      ddt_bias);
}
