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
// behind a single barrier.  Main loop: each thread owns 32 consecutive state
// entries of one row p (4 threads per row, 8 float4); the next head's state is
// loaded into registers before the current head's is stored, so every thread
// keeps 16 float4 loads in flight.
__global__ void __launch_bounds__(NT) m3_decode_step(DecArgs a) {
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
  // the first head's state is independent of the prologue: start streaming it now
  const int p = tid >> 2, part = tid & 3;
  float4 cur[8], nxt[8];
  auto state_row = [&](int hh) {
    return a.ssm + (((size_t)b * a.nh + h0 + hh) * P + p) * N + part * 32;
  };
  {
    const float4* src = reinterpret_cast<const float4*>(state_row(0));
#pragma unroll
    for (int q = 0; q < 8; ++q) cur[q] = src[q];
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
      const float4* src = reinterpret_cast<const float4*>(state_row(hh + 1));
#pragma unroll
      for (int q = 0; q < 8; ++q) nxt[q] = src[q];
    }
    const float dt = sDt[hh], dec = sDec[hh], sg = sSg[hh];
    const float cprev = (1.f - sg) * dt * dec * sVp[hh][p];
    const float ccur = sg * dt * sX[hh][p];
    const float* K = sK[hh];
    const float* Kp = sKp[hh];
    const float* Q = sQ[hh];
    float4* dst = reinterpret_cast<float4*>(state_row(hh));
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 hv = cur[q];
      const int n = part * 32 + q * 4;
      hv.x = dec * hv.x + cprev * Kp[n] + ccur * K[n];
      hv.y = dec * hv.y + cprev * Kp[n + 1] + ccur * K[n + 1];
      hv.z = dec * hv.z + cprev * Kp[n + 2] + ccur * K[n + 2];
      hv.w = dec * hv.w + cprev * Kp[n + 3] + ccur * K[n + 3];
      dst[q] = hv;
      acc += Q[n] * hv.x + Q[n + 1] * hv.y + Q[n + 2] * hv.z + Q[n + 3] * hv.w;
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (part == 0) {
      const int h = h0 + hh;
      const float z = sZ[hh][p];
      const float yv = (acc + a.D[h] * sX[hh][p]) * z * sigmoidf_(z);
      a.y[(size_t)b * a.d_inner + h * P + p] = __float2bfloat16(yv);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) cur[q] = nxt[q];
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
