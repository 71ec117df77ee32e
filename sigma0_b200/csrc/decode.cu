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

__global__ void __launch_bounds__(NT) m3_decode_step(DecArgs a) {
  __shared__ float sK[N], sQ[N], sKp[N], sX[P], sVp[P], sZ[P], sRed[2][8];
  __shared__ float sSc[4];
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bf16* row = a.proj + (size_t)b * a.ldp;
  const int off_B = 2 * a.d_inner, off_C = off_B + N, off_dt = off_C + N;
  const int off_A = off_dt + a.nh, off_tr = off_A + a.nh, off_ang = off_tr + a.nh;
  const size_t bh = (size_t)b * a.nh + h;
  // BCNorm sums (warps 0-3: B, 4-7: C)
  {
    float v = 0.f;
    if (tid < N) {
      float x = __bfloat162float(row[off_B + tid]);
      v = x * x;
    } else {
      float x = __bfloat162float(row[off_C + tid - N]);
      v = x * x;
    }
    v = warp_sum(v);
    if (lane == 0) sRed[warp >> 2][warp & 3] = v;
  }
  if (tid == 0) {
    float dt = softplusf_(__bfloat162float(row[off_dt + h]) + a.dt_bias[h]);
    float A = fminf(-softplusf_(__bfloat162float(row[off_A + h])), -a.A_floor);
    sSc[0] = dt;
    sSc[1] = __expf(A * dt);
    sSc[2] = sigmoidf_(__bfloat162float(row[off_tr + h]));
  }
  __syncthreads();
  const float dt = sSc[0], dec = sSc[1], sg = sSc[2];
  if (tid < N) {
    float ssb = sRed[0][0] + sRed[0][1] + sRed[0][2] + sRed[0][3];
    float ssc = sRed[1][0] + sRed[1][1] + sRed[1][2] + sRed[1][3];
    float rb = rsqrtf(ssb / N + a.eps), rc = rsqrtf(ssc / N + a.eps);
    sK[tid] = __bfloat162float(row[off_B + tid]) * rb * a.wB[tid] + a.Bb[h * N + tid];
    sQ[tid] = __bfloat162float(row[off_C + tid]) * rc * a.wC[tid] + a.Cb[h * N + tid];
    sKp[tid] = a.kprev[bh * N + tid];
  }
  if (tid < P) {
    sX[tid] = __bfloat162float(row[a.d_inner + h * P + tid]);
    sZ[tid] = __bfloat162float(row[h * P + tid]);
    sVp[tid] = a.vprev[bh * P + tid];
  }
  __syncthreads();
  if (tid < R) {   // angle state and rotation of the first 2R dims
    float th = a.ang[bh * R + tid] + tanhf(__bfloat162float(row[off_ang + tid])) * PI_F * dt;
    th = th - TWO_PI_F * floorf(th / TWO_PI_F);
    a.ang[bh * R + tid] = th;
    float sn, cs;
    sincosf(th, &sn, &cs);
    float k0 = sK[2 * tid], k1 = sK[2 * tid + 1], q0 = sQ[2 * tid], q1 = sQ[2 * tid + 1];
    sK[2 * tid] = k0 * cs - k1 * sn;
    sK[2 * tid + 1] = k0 * sn + k1 * cs;
    sQ[2 * tid] = q0 * cs - q1 * sn;
    sQ[2 * tid + 1] = q0 * sn + q1 * cs;
  }
  __syncthreads();
  // state rows: 4 threads per row p, 32 consecutive n each (float4 x 8)
  const int p = tid >> 2, part = tid & 3;
  float* hrow = a.ssm + (bh * P + p) * N + part * 32;
  const float cprev = (1.f - sg) * dt * dec * sVp[p];
  const float ccur = sg * dt * sX[p];
  float acc = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 hv = reinterpret_cast<float4*>(hrow)[q];
    int n = part * 32 + q * 4;
    hv.x = dec * hv.x + cprev * sKp[n] + ccur * sK[n];
    hv.y = dec * hv.y + cprev * sKp[n + 1] + ccur * sK[n + 1];
    hv.z = dec * hv.z + cprev * sKp[n + 2] + ccur * sK[n + 2];
    hv.w = dec * hv.w + cprev * sKp[n + 3] + ccur * sK[n + 3];
    reinterpret_cast<float4*>(hrow)[q] = hv;
    acc += sQ[n] * hv.x + sQ[n + 1] * hv.y + sQ[n + 2] * hv.z + sQ[n + 3] * hv.w;
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  if (part == 0) {
    float z = sZ[p];
    float yv = (acc + a.D[h] * sX[p]) * z * sigmoidf_(z);
    a.y[(size_t)b * a.d_inner + h * P + p] = __float2bfloat16(yv);
  }
  __syncthreads();
  if (tid < N) a.kprev[bh * N + tid] = sK[tid];
  if (tid < P) a.vprev[bh * P + tid] = sX[tid];
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
  s0::dec::m3_decode_step<<<dim3(nh, B), s0::dec::NT, 0, st>>>(a);
}
