// Mamba-3 recurrent decode step for sm_100a (autoregressive generation).
//
// One thread block per (head, book) advances the trapezoidal 3-term recurrence
// of the reference's __call_rnn__ (src/base_model/models/mamba3.py:466-578) by
// one token:
//   theta += tanh(a) * pi * dt  (mod 2pi);  K = rope(Bn + B_bias), Q = rope(Cn + C_bias)
//   h = e^{A dt} h + (1 - s) dt e^{A dt} (v_prev k_prev^T) + s dt (x K^T)
//   y = (Q . h + D x) * silu(z);            k_prev <- K, v_prev <- x
// The fp32 state (P x N per head) is read once and written once per token, so
// the step is bandwidth bound by construction; everything else (BCNorm, decay,
// RoPE) is recomputed in-block from the projection row.
#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace dec {

constexpr int N = 128, P = 64, R = 32, NT = 256;
constexpr float PI_F = 3.14159265358979323846f;
constexpr float TWO_PI_F = 6.28318530717958647692f;
using bf16 = __nv_bfloat16;

struct DecArgs {
  const bf16* proj;        // [B, ldp]
  int ldp, nh, d_inner;
  const float *wB, *wC, *dt_bias, *Bb, *Cb, *D;
  float A_floor, eps;
  float* ang;              // [B, nh, R]
  float* ssm;              // [B, nh, P, N]
  float* kprev;            // [B, nh, N]
  float* vprev;            // [B, nh, P]
  bf16* y;                 // [B, d_inner]
};

constexpr int HG = 8;   // heads per block: the per-token prologue is shared, state loads overlap

// One block per (group of HG heads, book).  The first head's state loads are
// issued before the prologue so their latency overlaps it.  Prologue: BCNorm of the token's B/C
// row (shared by all heads), per-head dt / decay / trapezoid gate, angle update
// and RoPE of K = Bn + B_bias[h], Q = Cn + C_bias[h], all into shared memory
// behind two barriers.  Main loop: each warp streams 8 rows of a head's state,
// one coalesced 512-byte row per instruction; the next head's state is loaded
// into registers before the current head's is stored, so every thread keeps
// 16 float4 loads in flight.
__global__ void __launch_bounds__(NT, 2) m3_decode_step(DecArgs a) {
  __shared__ float sBn[N], sCn[N];
  __shared__ float sK[HG][N], sQ[HG][N], sKp[HG][N];
  __shared__ float sX[HG][P], sVp[HG][P], sZ[HG][P];
  __shared__ float sDt[HG], sDec[HG], sSg[HG], sRed[2][4], sTh[HG][R];
  const int b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h0 = blockIdx.x * HG;
  const int nhg = min(HG, a.nh - h0);
  const bf16* row = a.proj + (size_t)b * a.ldp;
  const int off_B = 2 * a.d_inner, off_C = off_B + N, off_dt = off_C + N;
  const int off_A = off_dt + a.nh, off_tr = off_A + a.nh, off_ang = off_tr + a.nh;
  // the first head's state is independent of the prologue: start streaming it now.
  // Warp w owns rows 8w..8w+7 of the P x N state; lane l owns columns 4l..4l+3,
  // so each load/store instruction of a warp covers one contiguous 512-byte row.
  float4 cur[8], nxt[8];
  auto head_state = [&](int hh) {
    return reinterpret_cast<float4*>(a.ssm + (((size_t)b * a.nh + h0 + hh) * P + warp * 8) * N) + lane;
  };
  {
    const float4* src = head_state(0);
#pragma unroll
    for (int r = 0; r < 8; ++r) cur[r] = src[r * (N / 4)];
  }
  // BCNorm sums (warps 0-3: B, 4-7: C)
  float bc = __bfloat162float(row[(tid < N) ? off_B + tid : off_C + tid - N]);
  {
    float v = warp_sum(bc * bc);
    if (lane == 0) sRed[warp >> 2][warp & 3] = v;
  }
  if (tid < HG && tid < nhg) {
    const int h = h0 + tid;
    float dt = softplusf_(__bfloat162float(row[off_dt + h]) + a.dt_bias[h]);
    float A = fminf(-softplusf_(__bfloat162float(row[off_A + h])), -a.A_floor);
    sDt[tid] = dt;
    sDec[tid] = __expf(A * dt);
    sSg[tid] = sigmoidf_(__bfloat162float(row[off_tr + h]));
  }
  for (int i = tid; i < HG * P; i += NT) {
    const int hh = i / P, p = i % P;
    if (hh < nhg) {
      const int h = h0 + hh;
      const size_t bh = (size_t)b * a.nh + h;
      sX[hh][p] = __bfloat162float(row[a.d_inner + h * P + p]);
      sZ[hh][p] = __bfloat162float(row[h * P + p]);
      sVp[hh][p] = a.vprev[bh * P + p];
    }
  }
  __syncthreads();
  if (tid < N) {
    const float rb = rsqrtf((sRed[0][0] + sRed[0][1] + sRed[0][2] + sRed[0][3]) / N + a.eps);
    sBn[tid] = bc * rb * a.wB[tid];
  } else {
    const float rc = rsqrtf((sRed[1][0] + sRed[1][1] + sRed[1][2] + sRed[1][3]) / N + a.eps);
    sCn[tid - N] = bc * rc * a.wC[tid - N];
  }
  __syncthreads();
  // per head: biased K/Q, previous K, angle update + rotation of the first 2R dims
  for (int i = tid; i < HG * N; i += NT) {
    const int hh = i / N, n = i % N;
    if (hh < nhg) {
      const int h = h0 + hh;
      const size_t bh = (size_t)b * a.nh + h;
      sKp[hh][n] = a.kprev[bh * N + n];
      float k = sBn[n] + a.Bb[h * N + n], q = sCn[n] + a.Cb[h * N + n];
      if (n < 2 * R) {
        const int r = n >> 1;
        float th = a.ang[bh * R + r] + tanhf(__bfloat162float(row[off_ang + r])) * PI_F * sDt[hh];
        th = th - TWO_PI_F * floorf(th / TWO_PI_F);
        if ((n & 1) == 0) sTh[hh][r] = th;   // written back after the barrier below
        float sn, cs;
        sincosf(th, &sn, &cs);
        // partner element of the rotated pair
        const int m = n ^ 1;
        const float k2 = sBn[m] + a.Bb[h * N + m], q2 = sCn[m] + a.Cb[h * N + m];
        if ((n & 1) == 0) { k = k * cs - k2 * sn; q = q * cs - q2 * sn; }
        else { k = k2 * sn + k * cs; q = q2 * sn + q * cs; }
      }
      sK[hh][n] = k;
      sQ[hh][n] = q;
    }
  }
  __syncthreads();
  for (int hh = 0; hh < nhg; ++hh) {
    if (hh + 1 < nhg) {
      const float4* src = head_state(hh + 1);
#pragma unroll
      for (int r = 0; r < 8; ++r) nxt[r] = src[r * (N / 4)];
    }
    const float dt = sDt[hh], dec = sDec[hh], sg = sSg[hh];
    const float4 K = reinterpret_cast<const float4*>(sK[hh])[lane];
    const float4 Kp = reinterpret_cast<const float4*>(sKp[hh])[lane];
    const float4 Q = reinterpret_cast<const float4*>(sQ[hh])[lane];
    float4* dst = head_state(hh);
    float part[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int p = warp * 8 + r;
      const float cprev = (1.f - sg) * dt * dec * sVp[hh][p];
      const float ccur = sg * dt * sX[hh][p];
      float4 hv = cur[r];
      hv.x = dec * hv.x + cprev * Kp.x + ccur * K.x;
      hv.y = dec * hv.y + cprev * Kp.y + ccur * K.y;
      hv.z = dec * hv.z + cprev * Kp.z + ccur * K.z;
      hv.w = dec * hv.w + cprev * Kp.w + ccur * K.w;
      dst[r * (N / 4)] = hv;
      part[r] = Q.x * hv.x + Q.y * hv.y + Q.z * hv.z + Q.w * hv.w;
    }
    // transposed butterfly: 8 row sums over 32 lanes in 9 shuffles; lane l ends
    // with the full sum of row 4*b4 + 2*b3 + b2 (b_i = bit i of l)
    float q4[4], q2[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = u16 ? part[i] : part[i + 4], keep = u16 ? part[i + 4] : part[i];
      q4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = u8 ? q4[i] : q4[i + 2], keep = u8 ? q4[i + 2] : q4[i];
      q2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float acc;
    {
      const float send = u4 ? q2[0] : q2[1], keep = u4 ? q2[1] : q2[0];
      acc = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if ((lane & 3) == 0) {
      const int p = warp * 8 + (u16 ? 4 : 0) + (u8 ? 2 : 0) + (u4 ? 1 : 0);
      const int h = h0 + hh;
      const float z = sZ[hh][p];
      const float yv = (acc + a.D[h] * sX[hh][p]) * z * sigmoidf_(z);
      a.y[(size_t)b * a.d_inner + h * P + p] = __float2bfloat16(yv);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) cur[r] = nxt[r];
  }
  // the carries for the next token
  for (int i = tid; i < HG * R; i += NT) {
    const int hh = i / R, r = i % R;
    if (hh < nhg) a.ang[((size_t)b * a.nh + h0 + hh) * R + r] = sTh[hh][r];
  }
  for (int i = tid; i < HG * N; i += NT) {
    const int hh = i / N, n = i % N;
    if (hh < nhg) a.kprev[((size_t)b * a.nh + h0 + hh) * N + n] = sK[hh][n];
  }
  for (int i = tid; i < HG * P; i += NT) {
    const int hh = i / P, pp = i % P;
    if (hh < nhg) a.vprev[((size_t)b * a.nh + h0 + hh) * P + pp] = sX[hh][pp];
  }
}

// ---------------------------------------------------------------------------
// Several known tokens in one pass (the generator's computed time tokens): the
// state of each head is read once, advanced through T tokens in registers and
// written once, instead of T round trips through HBM.  Block = (group of HGM
// heads, book); per-token K/Q/x/z and scalars are prepared in shared memory.
// ---------------------------------------------------------------------------
constexpr int HGM = 4, TMAX = 8;

struct DecMultiArgs {
  DecArgs a;
  int T;                   // tokens (<= TMAX); proj rows are [B, T, ldp]
};

__global__ void __launch_bounds__(NT, 2) m3_decode_multi(DecMultiArgs ma) {
  const DecArgs& a = ma.a;
  const int T = ma.T;
  extern __shared__ float dsm[];
  float* sK = dsm;                                   // [T][HGM][N]
  float* sQ = sK + TMAX * HGM * N;                   // [T][HGM][N]
  float* sX = sQ + TMAX * HGM * N;                   // [T][HGM][P]
  float* sZ = sX + TMAX * HGM * P;                   // [T][HGM][P]
  float* sKp0 = sZ + TMAX * HGM * P;                 // [HGM][N]
  float* sVp0 = sKp0 + HGM * N;                      // [HGM][P]
  float* sDt = sVp0 + HGM * P;                       // [T][HGM]
  float* sDec = sDt + TMAX * HGM;
  float* sSg = sDec + TMAX * HGM;
  float* sBn = sSg + TMAX * HGM;                     // [T][N]
  float* sCn = sBn + TMAX * N;                       // [T][N]
  const int b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h0 = blockIdx.x * HGM;
  const int nhg = min(HGM, a.nh - h0);
  const int off_B = 2 * a.d_inner, off_C = off_B + N, off_dt = off_C + N;
  const int off_A = off_dt + a.nh, off_tr = off_A + a.nh, off_ang = off_tr + a.nh;
  // BCNorm per token: warp t (t < T) normalises B and C of token t
  for (int t = warp; t < T; t += NT / 32) {
    const bf16* row = a.proj + ((size_t)b * T + t) * a.ldp;
    float bv[4], cv[4], sb = 0.f, sc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      bv[i] = __bfloat162float(row[off_B + lane * 4 + i]);
      cv[i] = __bfloat162float(row[off_C + lane * 4 + i]);
      sb += bv[i] * bv[i];
      sc += cv[i] * cv[i];
    }
    sb = warp_sum(sb);
    sc = warp_sum(sc);
    const float rb = rsqrtf(sb / N + a.eps), rc = rsqrtf(sc / N + a.eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = lane * 4 + i;
      sBn[t * N + n] = bv[i] * rb * a.wB[n];
      sCn[t * N + n] = cv[i] * rc * a.wC[n];
    }
  }
  for (int i = tid; i < T * HGM; i += NT) {
    const int t = i / HGM, hh = i % HGM;
    if (hh < nhg) {
      const int h = h0 + hh;
      const bf16* row = a.proj + ((size_t)b * T + t) * a.ldp;
      const float dt = softplusf_(__bfloat162float(row[off_dt + h]) + a.dt_bias[h]);
      const float A = fminf(-softplusf_(__bfloat162float(row[off_A + h])), -a.A_floor);
      sDt[i] = dt;
      sDec[i] = __expf(A * dt);
      sSg[i] = sigmoidf_(__bfloat162float(row[off_tr + h]));
    }
  }
  for (int i = tid; i < T * HGM * P; i += NT) {
    const int t = i / (HGM * P), hh = (i / P) % HGM, p = i % P;
    if (hh < nhg) {
      const int h = h0 + hh;
      const bf16* row = a.proj + ((size_t)b * T + t) * a.ldp;
      sX[i] = __bfloat162float(row[a.d_inner + h * P + p]);
      sZ[i] = __bfloat162float(row[h * P + p]);
    }
  }
  for (int i = tid; i < HGM * N; i += NT) {
    const int hh = i / N, n = i % N;
    if (hh < nhg) sKp0[i] = a.kprev[((size_t)b * a.nh + h0 + hh) * N + n];
  }
  for (int i = tid; i < HGM * P; i += NT) {
    const int hh = i / P, p = i % P;
    if (hh < nhg) sVp0[i] = a.vprev[((size_t)b * a.nh + h0 + hh) * P + p];
  }
  __syncthreads();
  // angles: thread (hh, r) walks the T tokens; K/Q rotated per token
  if (tid < HGM * R) {
    const int hh = tid / R, r = tid % R;
    if (hh < nhg) {
      const size_t bh = (size_t)b * a.nh + h0 + hh;
      float th = a.ang[bh * R + r];
      for (int t = 0; t < T; ++t) {
        const bf16* row = a.proj + ((size_t)b * T + t) * a.ldp;
        th += tanhf(__bfloat162float(row[off_ang + r])) * PI_F * sDt[t * HGM + hh];
        th = th - TWO_PI_F * floorf(th / TWO_PI_F);
        float sn, cs;
        sincosf(th, &sn, &cs);
        const int h = h0 + hh;
        const float k0 = sBn[t * N + 2 * r] + a.Bb[h * N + 2 * r], k1 = sBn[t * N + 2 * r + 1] + a.Bb[h * N + 2 * r + 1];
        const float q0 = sCn[t * N + 2 * r] + a.Cb[h * N + 2 * r], q1 = sCn[t * N + 2 * r + 1] + a.Cb[h * N + 2 * r + 1];
        float* K = sK + (t * HGM + hh) * N;
        float* Q = sQ + (t * HGM + hh) * N;
        K[2 * r] = k0 * cs - k1 * sn;
        K[2 * r + 1] = k0 * sn + k1 * cs;
        Q[2 * r] = q0 * cs - q1 * sn;
        Q[2 * r + 1] = q0 * sn + q1 * cs;
      }
      a.ang[bh * R + r] = th;
    }
  }
  for (int i = tid; i < T * HGM * (N - 2 * R); i += NT) {
    const int t = i / (HGM * (N - 2 * R)), hh = (i / (N - 2 * R)) % HGM, n = 2 * R + i % (N - 2 * R);
    if (hh < nhg) {
      const int h = h0 + hh;
      sK[(t * HGM + hh) * N + n] = sBn[t * N + n] + a.Bb[h * N + n];
      sQ[(t * HGM + hh) * N + n] = sCn[t * N + n] + a.Cb[h * N + n];
    }
  }
  __syncthreads();
  for (int hh = 0; hh < nhg; ++hh) {
    const int h = h0 + hh;
    float4* st = reinterpret_cast<float4*>(a.ssm + (((size_t)b * a.nh + h) * P + warp * 8) * N) + lane;
    float4 cur[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) cur[r] = st[r * (N / 4)];
    for (int t = 0; t < T; ++t) {
      const int ti = t * HGM + hh;
      const float dt = sDt[ti], dec = sDec[ti], sg = sSg[ti];
      const float4 K = reinterpret_cast<const float4*>(sK + ti * N)[lane];
      const float4 Kp = t == 0 ? reinterpret_cast<const float4*>(sKp0 + hh * N)[lane]
                               : reinterpret_cast<const float4*>(sK + (ti - HGM) * N)[lane];
      const float4 Q = reinterpret_cast<const float4*>(sQ + ti * N)[lane];
      const float* Vp = t == 0 ? sVp0 + hh * P : sX + (ti - HGM) * P;
      const float* Xc = sX + ti * P;
      float part[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int p = warp * 8 + r;
        const float cprev = (1.f - sg) * dt * dec * Vp[p];
        const float ccur = sg * dt * Xc[p];
        float4 hv = cur[r];
        hv.x = dec * hv.x + cprev * Kp.x + ccur * K.x;
        hv.y = dec * hv.y + cprev * Kp.y + ccur * K.y;
        hv.z = dec * hv.z + cprev * Kp.z + ccur * K.z;
        hv.w = dec * hv.w + cprev * Kp.w + ccur * K.w;
        cur[r] = hv;
        part[r] = Q.x * hv.x + Q.y * hv.y + Q.z * hv.z + Q.w * hv.w;
      }
      float q4[4], q2[2];
      const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = u16 ? part[i] : part[i + 4], keep = u16 ? part[i + 4] : part[i];
        q4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = u8 ? q4[i] : q4[i + 2], keep = u8 ? q4[i + 2] : q4[i];
        q2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      float acc;
      {
        const float send = u4 ? q2[0] : q2[1], keep = u4 ? q2[1] : q2[0];
        acc = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if ((lane & 3) == 0) {
        const int p = warp * 8 + (u16 ? 4 : 0) + (u8 ? 2 : 0) + (u4 ? 1 : 0);
        const float z = sZ[ti * P + p];
        const float yv = (acc + a.D[h] * Xc[p]) * z * sigmoidf_(z);
        a.y[((size_t)b * T + t) * a.d_inner + h * P + p] = __float2bfloat16(yv);
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) st[r * (N / 4)] = cur[r];
  }
  // carries: the last token's rotated key and value
  for (int i = tid; i < HGM * N; i += NT) {
    const int hh = i / N, n = i % N;
    if (hh < nhg) a.kprev[((size_t)b * a.nh + h0 + hh) * N + n] = sK[((T - 1) * HGM + hh) * N + n];
  }
  for (int i = tid; i < HGM * P; i += NT) {
    const int hh = i / P, p = i % P;
    if (hh < nhg) a.vprev[((size_t)b * a.nh + h0 + hh) * P + p] = sX[((T - 1) * HGM + hh) * P + p];
  }
}

}  // namespace dec
}  // namespace s0

void m3_decode_step_launch(const void* proj, int B, int ldp, int nh, const float* wB, const float* wC,
                           const float* dt_bias, const float* Bb, const float* Cb, const float* D, float A_floor,
                           float eps, float* ang, float* ssm, float* kprev, float* vprev, void* y,
                           cudaStream_t st) {
  s0::dec::DecArgs a;
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.nh = nh;
  a.d_inner = nh * s0::dec::P;
  a.wB = wB; a.wC = wC; a.dt_bias = dt_bias; a.Bb = Bb; a.Cb = Cb; a.D = D;
  a.A_floor = A_floor; a.eps = eps;
  a.ang = ang; a.ssm = ssm; a.kprev = kprev; a.vprev = vprev;
  a.y = reinterpret_cast<__nv_bfloat16*>(y);
  s0::dec::m3_decode_step<<<dim3((nh + s0::dec::HG - 1) / s0::dec::HG, B), s0::dec::NT, 0, st>>>(a);
}

void m3_decode_multi_launch(const void* proj, int B, int T, int ldp, int nh, const float* wB, const float* wC,
                            const float* dt_bias, const float* Bb, const float* Cb, const float* D, float A_floor,
                            float eps, float* ang, float* ssm, float* kprev, float* vprev, void* y,
                            cudaStream_t st) {
  s0::dec::DecMultiArgs ma;
  s0::dec::DecArgs& a = ma.a;
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.nh = nh;
  a.d_inner = nh * s0::dec::P;
  a.wB = wB; a.wC = wC; a.dt_bias = dt_bias; a.Bb = Bb; a.Cb = Cb; a.D = D;
  a.A_floor = A_floor; a.eps = eps;
  a.ang = ang; a.ssm = ssm; a.kprev = kprev; a.vprev = vprev;
  a.y = reinterpret_cast<__nv_bfloat16*>(y);
  ma.T = T;
  using namespace s0::dec;
  const size_t smem = sizeof(float) * (2 * TMAX * HGM * N + 2 * TMAX * HGM * P + HGM * N + HGM * P +
                                       3 * TMAX * HGM + 2 * TMAX * N);
  cudaFuncSetAttribute(m3_decode_multi, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  m3_decode_multi<<<dim3((nh + HGM - 1) / HGM, B), NT, smem, st>>>(ma);
}
