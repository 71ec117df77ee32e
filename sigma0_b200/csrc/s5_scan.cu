// Complex diagonal linear recurrence of the S5 layer, forward and backward, for sm_100a.
//
// x_t = lam * x_{t-1} + Bu_t over (B, L, P) complex64 (the reference's associative scan,
// src/base_model/models/ssm.py:78-111; K21).  The sequence is cut into chunks of T = 64
// steps and scanned in three passes, each with one thread per (batch, chunk, channel)
// so consecutive threads read consecutive channels:
//   1. chunk-local end values from a zero start;
//   2. per (batch, channel), the carries entering every chunk: c_{k+1} = lam^T c_k + end_k
//      (lam^T by repeated squaring; x0 is the first carry);
//   3. the chunk re-scanned from its carry, every x_t written (and the final state).
// The backward is the same in reverse time with conj(lam) (PyTorch's conjugate
// convention for complex gradients): G_t = dxs_t + conj(lam) G_{t+1}, dBu_t = G_t,
// dlam = sum_t G_t conj(x_{t-1}) (block partials added with atomics), dx0 = conj(lam) G_0.
#include <cuda_runtime.h>

#include "launchers.h"

namespace s0 {
namespace s5 {

constexpr int T = 64, NT = 256;
constexpr int U = 8;   // steps whose loads are issued together (they do not depend on the recurrence)

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cfma(float2 a, float2 b, float2 c) {   // a * b + c
  return make_float2(fmaf(a.x, b.x, fmaf(-a.y, b.y, c.x)), fmaf(a.x, b.y, fmaf(a.y, b.x, c.y)));
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cpow(float2 a, int n) {                // a^n, n >= 0
  float2 r = make_float2(1.f, 0.f);
  while (n) {
    if (n & 1) r = cmul(r, a);
    a = cmul(a, a);
    n >>= 1;
  }
  return r;
}

// thread -> (b, chunk, p) with p fastest
__device__ __forceinline__ bool index(const S5Args& a, long& b, int& c, int& p) {
  const long i = (long)blockIdx.x * NT + threadIdx.x;
  const long per_b = (long)a.nchunk * a.P;
  if (i >= a.B * per_b) return false;
  b = i / per_b;
  c = (int)((i % per_b) / a.P);
  p = (int)(i % a.P);
  return true;
}

__global__ void __launch_bounds__(NT) s5_fwd_local_k(S5Args a) {
  long b;
  int c, p;
  if (!index(a, b, c, p)) return;
  const float2 lam = a.lam[p];
  const int t0 = c * T, t1 = min(a.L, t0 + T);
  const float2* bu = a.bu + (b * a.L) * a.P + p;
  float2 x = make_float2(0.f, 0.f);
  for (int t = t0; t < t1; t += U) {
    float2 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = t + u < t1 ? bu[(long)(t + u) * a.P] : make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (t + u < t1) x = cfma(lam, x, v[u]);
  }
  a.part[(b * a.nchunk + c) * a.P + p] = x;
}

// carries: fwd (dir 0): c_0 = x0, c_{k+1} = lam^T c_k + end_k;
//          bwd (dir 1): R_last = 0, R_{k-1} = end_k + conj(lam)^{len_k} R_k
__global__ void __launch_bounds__(NT) s5_carry_k(S5Args a, int dir) {
  const long i = (long)blockIdx.x * NT + threadIdx.x;
  if (i >= (long)a.B * a.P) return;
  const long b = i / a.P;
  const int p = (int)(i % a.P);
  const float2 lam = dir ? cconj(a.lam[p]) : a.lam[p];
  const float2 lT = cpow(lam, T);
  float2* part = a.part + b * a.nchunk * a.P + p;
  if (!dir) {
    float2 cr = a.x0 ? a.x0[b * a.P + p] : make_float2(0.f, 0.f);
    for (int c = 0; c < a.nchunk; ++c) {
      const float2 e = part[(long)c * a.P];
      part[(long)c * a.P] = cr;                                   // in place: end -> carry in
      cr = cfma(lT, cr, e);
    }
  } else {
    float2 r = make_float2(0.f, 0.f);
    for (int c = a.nchunk - 1; c >= 0; --c) {
      const float2 e = part[(long)c * a.P];
      part[(long)c * a.P] = r;
      const int len = min(a.L, (c + 1) * T) - c * T;
      r = cfma(len == T ? lT : cpow(lam, len), r, e);
    }
  }
}

__global__ void __launch_bounds__(NT) s5_fwd_apply_k(S5Args a) {
  long b;
  int c, p;
  if (!index(a, b, c, p)) return;
  const float2 lam = a.lam[p];
  const int t0 = c * T, t1 = min(a.L, t0 + T);
  const long base = (b * a.L) * a.P + p;
  float2 x = a.part[(b * a.nchunk + c) * a.P + p];
  for (int t = t0; t < t1; t += U) {
    float2 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = t + u < t1 ? a.bu[base + (long)(t + u) * a.P] : make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (t + u < t1) {
        x = cfma(lam, x, v[u]);
        a.xs[base + (long)(t + u) * a.P] = x;
      }
  }
  if (t1 == a.L) a.xlast[b * a.P + p] = x;
}

__global__ void __launch_bounds__(NT) s5_bwd_local_k(S5Args a) {
  long b;
  int c, p;
  if (!index(a, b, c, p)) return;
  const float2 lc = cconj(a.lam[p]);
  const int t0 = c * T, t1 = min(a.L, t0 + T);
  const long base = (b * a.L) * a.P + p;
  float2 g = make_float2(0.f, 0.f);
  const float2 e = (t1 == a.L && a.dxlast) ? a.dxlast[b * a.P + p] : make_float2(0.f, 0.f);
  for (int t = t1 - 1; t >= t0; t -= U) {
    float2 d[U];
#pragma unroll
    for (int u = 0; u < U; ++u) d[u] = t - u >= t0 ? a.dxs[base + (long)(t - u) * a.P] : make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (t - u >= t0) {
        if (t - u == a.L - 1) {
          d[u].x += e.x;
          d[u].y += e.y;
        }
        g = cfma(lc, g, d[u]);
      }
  }
  a.part[(b * a.nchunk + c) * a.P + p] = g;
}

__global__ void __launch_bounds__(NT) s5_bwd_apply_k(S5Args a) {
  long b;
  int c, p;
  if (!index(a, b, c, p)) return;
  const float2 lam = a.lam[p], lc = cconj(lam);
  const int t0 = c * T, t1 = min(a.L, t0 + T);
  const long base = (b * a.L) * a.P + p;
  float2 g = a.part[(b * a.nchunk + c) * a.P + p];
  float2 dl = make_float2(0.f, 0.f);
  const float2 e = (t1 == a.L && a.dxlast) ? a.dxlast[b * a.P + p] : make_float2(0.f, 0.f);
  const float2 x0 = a.x0 ? a.x0[b * a.P + p] : make_float2(0.f, 0.f);
  for (int t = t1 - 1; t >= t0; t -= U) {
    float2 d[U], xp[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int tt = t - u;
      d[u] = tt >= t0 ? a.dxs[base + (long)tt * a.P] : make_float2(0.f, 0.f);
      xp[u] = tt >= t0 && tt > 0 ? a.xs[base + (long)(tt - 1) * a.P] : x0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int tt = t - u;
      if (tt >= t0) {
        if (tt == a.L - 1) {
          d[u].x += e.x;
          d[u].y += e.y;
        }
        g = cfma(lc, g, d[u]);
        a.dbu[base + (long)tt * a.P] = g;
        dl = cfma(g, cconj(xp[u]), dl);
      }
    }
  }
  atomicAdd(&a.dlam[p].x, dl.x);
  atomicAdd(&a.dlam[p].y, dl.y);
  if (t0 == 0 && a.dx0) a.dx0[b * a.P + p] = cmul(lc, g);
}

}  // namespace s5
}  // namespace s0

int s5_scan_launch(const S5Args& a, bool bwd, cudaStream_t st) {
  using namespace s0::s5;
  if (a.B <= 0 || a.L <= 0 || a.P <= 0) return 0;
  const long n = (long)a.B * a.nchunk * a.P;
  const unsigned g1 = (unsigned)((n + NT - 1) / NT), g2 = (unsigned)(((long)a.B * a.P + NT - 1) / NT);
  if (!bwd) {
    s5_fwd_local_k<<<g1, NT, 0, st>>>(a);
    s5_carry_k<<<g2, NT, 0, st>>>(a, 0);
    s5_fwd_apply_k<<<g1, NT, 0, st>>>(a);
  } else {
    s5_bwd_local_k<<<g1, NT, 0, st>>>(a);
    s5_carry_k<<<g2, NT, 0, st>>>(a, 1);
    s5_bwd_apply_k<<<g1, NT, 0, st>>>(a);
  }
  return (int)cudaGetLastError();
}
