// Fused row-wise kernels of the residual block, the loss and the optimizer (sm_100a).
//
//  ln_fwd / ln_bwd          LayerNorm (fp32 residual in, bf16 out) and its backward fused
//                           with the residual add; scale/bias grads reduced per block
//  rms_fwd / rms_bwd        RMSNorm over d_inner (bf16 in/out), the out_norm of Mamba3
//  gelu_fwd                 tanh-GELU (the reference uses flax's approximate gelu)
//  glu_res_fwd / _bwd       out = x + g * sigmoid(h + b)  (half_glu1 gate + residual)
//  gelu_bwd                 d o = (dg_gate + dg_mm) * gelu'(o)
//  ce_fwd_bwd               per-row log-softmax cross-entropy and its logit gradient,
//                           written in place over the bf16 logits
//  sumsq / adam_step        global-norm clip + Adam/AdamW update of a flat fp32 buffer,
//                           writing the bf16 compute copy in the same pass
//
// The GELU tanh approximation uses the published constants of Hendrycks & Gimpel
// (sqrt(2/pi), 0.044715).  Row kernels are one warp per row; column (parameter)
// reductions accumulate per warp over a grid-stride row loop, then one atomicAdd
// per column per warp.
#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace ops {

using bf16 = __nv_bfloat16;
using s0::gelu_t;
using s0::gelu_t_grad;

// Max 64 columns per lane (D <= 2048).
constexpr int MAXV = 64;

// Reduce per-warp column partials across the warps of a block through shared memory,
// then one atomicAdd per column per block.  `vals[i]` is this lane's partial for
// column lane + 32*i (VPL entries); `smem` holds blockDim/32 * 32 * VPL floats.
template <int VPL>
S0_DEV void block_col_atomic(float* vals, float* smem, float* out, int D) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < VPL; ++i) smem[(w * VPL + i) * 32 + lane] = vals[i];
  __syncthreads();
  for (int c = threadIdx.x; c < VPL * 32; c += blockDim.x) {
    int i = c >> 5, l = c & 31;
    float s = 0.f;
    for (int k = 0; k < nw; ++k) s += smem[(k * VPL + i) * 32 + l];
    int col = l + 32 * i;
    if (col < D) atomicAdd(&out[col], s);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// LayerNorm forward: x fp32 [T, D] -> y bf16, mean/rstd fp32 [T]
// ---------------------------------------------------------------------------
template <int VPL>
__global__ void ln_fwd_k(const float* __restrict__ x, const float* __restrict__ w,
                         const float* __restrict__ b, bf16* __restrict__ y, float* __restrict__ mean,
                         float* __restrict__ rstd, int T, int D, float eps) {
  int lane = threadIdx.x & 31;
  int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int nw = (gridDim.x * blockDim.x) >> 5;
  for (int row = gw; row < T; row += nw) {
    const float* xr = x + (size_t)row * D;
    float v[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      int c = lane + 32 * i;
      v[i] = c < D ? xr[c] : 0.f;
      s += v[i];
    }
    s = warp_sum(s);
    float mu = s / D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      int c = lane + 32 * i;
      float d = c < D ? v[i] - mu : 0.f;
      q += d * d;
    }
    q = warp_sum(q);
    float r = rsqrtf(q / D + eps);
    bf16* yr = y + (size_t)row * D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      int c = lane + 32 * i;
      if (c < D) yr[c] = __float2bfloat16((v[i] - mu) * r * w[c] + b[c]);
    }
    if (lane == 0) { mean[row] = mu; rstd[row] = r; }
  }
}

// Column reductions (dgamma, dbeta, dbias) without atomics: every warp
// accumulates its rows' contributions in its own shared-memory row (no
// conflicts: a column belongs to one lane), the block sums its warps into one
// partial row of `part`, and col_sum_k adds the blocks' partial rows in a fixed
// order (deterministic).  Row data moves as float4 / 4 x bf16.
constexpr int CB_NT = 256;

__device__ __forceinline__ float4 ld_bf16x4(const bf16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st_bf16x4(bf16* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
}
__device__ __forceinline__ void add4(float* p, float4 v) {
  float4 o = *reinterpret_cast<float4*>(p);
  o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
  *reinterpret_cast<float4*>(p) = o;
}

// LayerNorm backward fused with the residual: dx = dres + LN'(dy); per-block
// partial rows of dw and db go to part[block][2][D].  J float4 chunks per lane.
template <int J>
__global__ void __launch_bounds__(CB_NT)
    ln_bwd_k(const bf16* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean,
             const float* __restrict__ rstd, const float* __restrict__ w, const float* __restrict__ dres,
             float* __restrict__ dx, float* __restrict__ part, int T, int D) {
  extern __shared__ __align__(16) float red_smem[];   // [8][2][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* sw = red_smem + (size_t)wid * 2 * D;
  float* sb = sw + D;
  for (int c = lane * 4; c < 2 * D; c += 128) *reinterpret_cast<float4*>(sw + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  const int gw = blockIdx.x * (CB_NT / 32) + wid, nw = gridDim.x * (CB_NT / 32);
  for (int row = gw; row < T; row += nw) {
    const size_t o = (size_t)row * D;
    const float mu = mean[row], r = rstd[row];
    float4 xh[J], gw_[J];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        const float4 xv = *reinterpret_cast<const float4*>(x + o + c);
        const float4 g = ld_bf16x4(dy + o + c);
        const float4 wv = *reinterpret_cast<const float4*>(w + c);
        xh[j] = make_float4((xv.x - mu) * r, (xv.y - mu) * r, (xv.z - mu) * r, (xv.w - mu) * r);
        gw_[j] = make_float4(g.x * wv.x, g.y * wv.y, g.z * wv.z, g.w * wv.w);
        s1 += gw_[j].x + gw_[j].y + gw_[j].z + gw_[j].w;
        s2 += gw_[j].x * xh[j].x + gw_[j].y * xh[j].y + gw_[j].z * xh[j].z + gw_[j].w * xh[j].w;
        add4(sw + c, make_float4(g.x * xh[j].x, g.y * xh[j].y, g.z * xh[j].z, g.w * xh[j].w));
        add4(sb + c, g);
      }
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        float4 rv = dres ? *reinterpret_cast<const float4*>(dres + o + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        rv.x += r * (gw_[j].x - s1 - xh[j].x * s2);
        rv.y += r * (gw_[j].y - s1 - xh[j].y * s2);
        rv.z += r * (gw_[j].z - s1 - xh[j].z * s2);
        rv.w += r * (gw_[j].w - s1 - xh[j].w * s2);
        *reinterpret_cast<float4*>(dx + o + c) = rv;
      }
    }
  }
  __syncthreads();
  float* dst = part + (size_t)blockIdx.x * 2 * D;
  for (int c = threadIdx.x; c < 2 * D; c += CB_NT) {
    float t = 0.f;
    for (int k = 0; k < CB_NT / 32; ++k) t += red_smem[(size_t)k * 2 * D + c];
    dst[c] = t;
  }
}

// LayerNorm backward, pipelined (same math as ln_bwd_k): each warp stages its next
// row (x fp32, dy bf16, dres fp32) in shared memory with cp.async while computing the
// current one.  LB_NW warps per block, one block per SM; dw / db partials in registers
// (a lane owns its columns), summed over the warps through shared memory at the end.
// D <= 1024, D % 4 == 0.
constexpr int LB_NW = 10;
__global__ void __launch_bounds__(LB_NW * 32, 1)
    ln_bwd_pipe_k(const bf16* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean,
                  const float* __restrict__ rstd, const float* __restrict__ w, const float* __restrict__ dres,
                  float* __restrict__ dx, float* __restrict__ part, int T, int D) {
  constexpr int J = 8;                                             // float4 chunks per lane (D <= 1024)
  extern __shared__ __align__(16) unsigned char lb_smem[];
  float* sw = reinterpret_cast<float*>(lb_smem);                   // [D]
  float* stage = sw + 3 * D;                                       // [LB_NW][2][x D | dres D | dy D/2]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int SZ = 2 * D + D / 2;                                    // floats per staged row
  for (int c = threadIdx.x; c < D; c += blockDim.x) sw[c] = w[c];
  float4 aw[J], ab[J];
#pragma unroll
  for (int j = 0; j < J; ++j) aw[j] = ab[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  float* my = stage + (size_t)wid * 2 * SZ;
  const int gw = blockIdx.x * LB_NW + wid, nw = gridDim.x * LB_NW;
  auto issue = [&](int row, int buf) {
    float* bx = my + (size_t)buf * SZ;
    float* br = bx + D;
    bf16* bg = reinterpret_cast<bf16*>(br + D);
    const size_t o = (size_t)row * D;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        cp_async16(bx + c, x + o + c);
        if (dres) cp_async16(br + c, dres + o + c);
        cp_async8(bg + c, dy + o + c);
      }
    }
  };
  __syncthreads();
  int buf = 0;
  float mu_n = 0.f, r_n = 0.f;
  if (gw < T) { issue(gw, 0); mu_n = mean[gw]; r_n = rstd[gw]; }
  cp_async_commit();
  for (int row = gw; row < T; row += nw) {
    const float mu = mu_n, r = r_n;
    const int nxt = row + nw;
    if (nxt < T) { issue(nxt, buf ^ 1); mu_n = mean[nxt]; r_n = rstd[nxt]; }
    cp_async_commit();
    cp_async_wait_group<1>();
    const float* bx = my + (size_t)buf * SZ;
    const float* br = bx + D;
    const bf16* bg = reinterpret_cast<const bf16*>(br + D);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        const float4 xv = *reinterpret_cast<const float4*>(bx + c);
        const float4 g = ld_bf16x4(bg + c);
        const float4 wv = *reinterpret_cast<const float4*>(sw + c);
        const float h0 = (xv.x - mu) * r, h1 = (xv.y - mu) * r, h2 = (xv.z - mu) * r, h3 = (xv.w - mu) * r;
        const float a0 = g.x * wv.x, a1 = g.y * wv.y, a2 = g.z * wv.z, a3 = g.w * wv.w;
        s1 += a0 + a1 + a2 + a3;
        s2 += a0 * h0 + a1 * h1 + a2 * h2 + a3 * h3;
        aw[j].x += g.x * h0; aw[j].y += g.y * h1; aw[j].z += g.z * h2; aw[j].w += g.w * h3;
        ab[j].x += g.x; ab[j].y += g.y; ab[j].z += g.z; ab[j].w += g.w;
      }
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
    const size_t o = (size_t)row * D;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        const float4 xv = *reinterpret_cast<const float4*>(bx + c);
        const float4 g = ld_bf16x4(bg + c);
        const float4 wv = *reinterpret_cast<const float4*>(sw + c);
        float4 rv = dres ? *reinterpret_cast<const float4*>(br + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        rv.x += r * (g.x * wv.x - s1 - (xv.x - mu) * r * s2);
        rv.y += r * (g.y * wv.y - s1 - (xv.y - mu) * r * s2);
        rv.z += r * (g.z * wv.z - s1 - (xv.z - mu) * r * s2);
        rv.w += r * (g.w * wv.w - s1 - (xv.w - mu) * r * s2);
        *reinterpret_cast<float4*>(dx + o + c) = rv;
      }
    }
    buf ^= 1;
  }
  cp_async_wait_all();
  __syncthreads();
  float* red = stage;                                              // [LB_NW][2][D]
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = 4 * (lane + 32 * j);
    if (c < D) {
      *reinterpret_cast<float4*>(red + (size_t)wid * 2 * D + c) = aw[j];
      *reinterpret_cast<float4*>(red + (size_t)wid * 2 * D + D + c) = ab[j];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < LB_NW; ++k) t += red[(size_t)k * 2 * D + c];
    part[(size_t)blockIdx.x * 2 * D + c] = t;
  }
}

// out_s[c] = sum over blocks of part[block][s][c], s < sets.  Block = 32 columns x
// 8 row slices (coalesced along columns); fixed summation order (deterministic).
__global__ void __launch_bounds__(256) col_sum_k(const float* __restrict__ part, int nblk, int sets, int D,
                                                 float* __restrict__ out0, float* __restrict__ out1) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + tx;
  const int W = sets * D;
  float t = 0.f;
  if (i < W)
    for (int b = ty; b < nblk; b += 8) t += part[(size_t)b * W + i];
  red[ty][tx] = t;
  __syncthreads();
  if (ty == 0 && i < W) {
    float u = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) u += red[k][tx];
    const int sset = i / D, c = i % D;
    (sset == 0 ? out0 : out1)[c] = u;
  }
}

// ---------------------------------------------------------------------------
// RMSNorm over bf16 rows (out_norm): y = x * rsqrt(mean(x^2)+eps) * w
// ---------------------------------------------------------------------------
// One warp per row; PER 16-byte chunks per lane hold the whole row in registers, so
// all of a row's loads are in flight at once (D <= 256 * PER).  w must be 16-byte aligned.
template <int PER>
__global__ void __launch_bounds__(256, 2) rms_fwd_k(const bf16* __restrict__ x, const float* __restrict__ w,
                                                 bf16* __restrict__ y, float* __restrict__ rstd, int T, int D,
                                                 float eps) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int nv = D / 8;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int row = gw; row < T; row += nw) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
    uint4 u[PER];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      u[j] = c < nv ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const uint32_t a[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) { const float2 f = unpack_bf16(a[k]); s += f.x * f.x + f.y * f.y; }
    }
    const float r = rsqrtf(warp_sum(s) / D + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t a[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16(a[k]);
          o[k] = pack_bf16(f.x * r * ws[2 * k], f.y * r * ws[2 * k + 1]);
        }
        yr[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (lane == 0) rstd[row] = r;
  }
}

// RMSNorm backward: one warp per row with the row of x and dy in registers (all loads
// in flight together); dw column partials accumulate in the warp's own shared-memory
// row (a column belongs to one lane, no conflicts) and each block writes one partial
// row, summed by col_sum_k.  w must be 16-byte aligned.
template <int PER>
__global__ void __launch_bounds__(256, 2) rms_bwd_k(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                 const float* __restrict__ w, const float* __restrict__ rstd,
                                                 bf16* __restrict__ dx, float* __restrict__ dw, int T, int D) {
  extern __shared__ __align__(16) float red_smem[];   // [8][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int nv = D / 8;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float* sw = red_smem + (size_t)wid * D;
  for (int c = lane * 4; c < D; c += 128) *reinterpret_cast<float4*>(sw + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  for (int row = gw; row < T; row += nw) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * D);
    const float r = rstd[row];
    uint4 ux[PER], ug[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      const bool ok = c < nv;
      ux[j] = ok ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
      ug[j] = ok ? gr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux[j].x, ux[j].y, ux[j].z, ux[j].w}, ag[4] = {ug[j].x, ug[j].y, ug[j].z, ug[j].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          m += fg.x * ws[2 * k] * fx.x + fg.y * ws[2 * k + 1] * fx.y;
        }
      }
    }
    m = warp_sum(m) / D;
    const float r3m = r * r * r * m;
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux[j].x, ux[j].y, ux[j].z, ux[j].w}, ag[4] = {ug[j].x, ug[j].y, ug[j].z, ug[j].w};
        uint32_t o[4];
        float cw[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          o[k] = pack_bf16(r * fg.x * ws[2 * k] - fx.x * r3m, r * fg.y * ws[2 * k + 1] - fx.y * r3m);
          cw[2 * k] = fg.x * fx.x * r;
          cw[2 * k + 1] = fg.y * fx.y * r;
        }
        dr[c] = make_uint4(o[0], o[1], o[2], o[3]);
        add4(sw + c * 8, make_float4(cw[0], cw[1], cw[2], cw[3]));
        add4(sw + c * 8 + 4, make_float4(cw[4], cw[5], cw[6], cw[7]));
      }
    }
  }
  __syncthreads();
  const int nwb = blockDim.x >> 5;
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < nwb; ++k) t += red_smem[(size_t)k * D + col];
    dw[(size_t)blockIdx.x * D + col] = t;   // this block's partial row (dw is the partial buffer)
  }
}

// RMSNorm for wide rows (2048 < D <= 1024 * PER): one 128-thread block per row, each
// thread holding PER 16-byte chunks (columns tid + 128 j), the row sum reduced through
// four shared-memory slots.  The backward keeps each thread's dw columns in registers
// across its rows and writes one partial row per block for col_sum_k.
constexpr int RW_NT = 128;
template <int PER>
__global__ void __launch_bounds__(RW_NT) rms_fwd_wide_k(const bf16* __restrict__ x, const float* __restrict__ w,
                                                      bf16* __restrict__ y, float* __restrict__ rstd, int T, int D,
                                                      float eps) {
  __shared__ float red[RW_NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nv = D / 8;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
    uint4 u[PER];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = tid + RW_NT * j;
      u[j] = c < nv ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const uint32_t a[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) { const float2 f = unpack_bf16(a[k]); s += f.x * f.x + f.y * f.y; }
    }
    s = warp_sum(s);
    if (lane == 0) red[wid] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < RW_NT / 32; ++k) tot += red[k];
    __syncthreads();                       // red is rewritten by the next row
    const float r = rsqrtf(tot / D + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = tid + RW_NT * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t a[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16(a[k]);
          o[k] = pack_bf16(f.x * r * ws[2 * k], f.y * r * ws[2 * k + 1]);
        }
        yr[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (tid == 0) rstd[row] = r;
  }
}

template <int PER>
__global__ void __launch_bounds__(RW_NT) rms_bwd_wide_k(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                      const float* __restrict__ w, const float* __restrict__ rstd,
                                                      bf16* __restrict__ dx, float* __restrict__ part, int T,
                                                      int D) {
  __shared__ float red[RW_NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nv = D / 8;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float aw[PER * 8];
#pragma unroll
  for (int i = 0; i < PER * 8; ++i) aw[i] = 0.f;
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * D);
    const float r = rstd[row];
    uint4 ux[PER], ug[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = tid + RW_NT * j;
      const bool ok = c < nv;
      ux[j] = ok ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
      ug[j] = ok ? gr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = tid + RW_NT * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux[j].x, ux[j].y, ux[j].z, ux[j].w}, ag[4] = {ug[j].x, ug[j].y, ug[j].z, ug[j].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          m += fg.x * ws[2 * k] * fx.x + fg.y * ws[2 * k + 1] * fx.y;
        }
      }
    }
    m = warp_sum(m);
    if (lane == 0) red[wid] = m;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < RW_NT / 32; ++k) tot += red[k];
    __syncthreads();
    const float r3m = r * r * r * (tot / D);
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = tid + RW_NT * j;
      if (c < nv) {
        const float4 wa = w4[2 * c], wb = w4[2 * c + 1];
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux[j].x, ux[j].y, ux[j].z, ux[j].w}, ag[4] = {ug[j].x, ug[j].y, ug[j].z, ug[j].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          o[k] = pack_bf16(r * fg.x * ws[2 * k] - fx.x * r3m, r * fg.y * ws[2 * k + 1] - fx.y * r3m);
          aw[j * 8 + 2 * k] += fg.x * fx.x * r;
          aw[j * 8 + 2 * k + 1] += fg.y * fx.y * r;
        }
        dr[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  float* pr = part + (size_t)blockIdx.x * D;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int c = tid + RW_NT * j;
    if (c < nv) {
      *reinterpret_cast<float4*>(pr + c * 8) = make_float4(aw[j * 8], aw[j * 8 + 1], aw[j * 8 + 2], aw[j * 8 + 3]);
      *reinterpret_cast<float4*>(pr + c * 8 + 4) =
          make_float4(aw[j * 8 + 4], aw[j * 8 + 5], aw[j * 8 + 6], aw[j * 8 + 7]);
    }
  }
}

// RMSNorm backward, pipelined: each warp stages its NEXT row of x and dy in shared
// memory with cp.async while it computes the current one, so every warp always has a
// row in flight (the register version issues one row's loads, waits, computes, and
// only then loads the next).  12 warps per block, one block per SM:
//   stage [12 warps][2 buffers][x | dy][D] bf16 + w [D] + dw accumulators [D] fp32.
// dw partials accumulate in registers (a lane owns its columns for every row), then the
// block's warps are summed through shared memory into one partial row for col_sum_k.
constexpr int RB_NW = 12;
template <int PER>
__global__ void __launch_bounds__(RB_NW * 32, 1)
    rms_bwd_pipe_k(const bf16* __restrict__ dy, const bf16* __restrict__ x, const float* __restrict__ w,
                   const float* __restrict__ rstd, bf16* __restrict__ dx, float* __restrict__ part, int T, int D) {
  extern __shared__ __align__(16) unsigned char rb_smem[];
  float* sw = reinterpret_cast<float*>(rb_smem);                 // [D]
  float* sred = sw + D;                                          // [D] (unused until the end)
  bf16* stage = reinterpret_cast<bf16*>(sred + D);               // [RB_NW][2][2][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nv = D / 8;
  for (int c = threadIdx.x; c < D; c += blockDim.x) sw[c] = w[c];
  float aw[PER * 8];
#pragma unroll
  for (int i = 0; i < PER * 8; ++i) aw[i] = 0.f;
  bf16* my = stage + (size_t)wid * 4 * D;
  const int gw = blockIdx.x * RB_NW + wid, nw = gridDim.x * RB_NW;
  auto issue = [&](int row, int buf) {
    bf16* bx = my + (size_t)buf * 2 * D;
    bf16* bg = bx + D;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        cp_async16(bx + c * 8, x + (size_t)row * D + c * 8);
        cp_async16(bg + c * 8, dy + (size_t)row * D + c * 8);
      }
    }
  };
  __syncthreads();
  int buf = 0;
  float r_next = 0.f;
  if (gw < T) { issue(gw, 0); r_next = rstd[gw]; }
  cp_async_commit();
  for (int row = gw; row < T; row += nw) {
    const float r = r_next;
    const int nxt = row + nw;
    if (nxt < T) { issue(nxt, buf ^ 1); r_next = rstd[nxt]; }
    cp_async_commit();
    cp_async_wait_group<1>();        // this row's copies (this lane's own chunks) are in
    const bf16* bx = my + (size_t)buf * 2 * D;
    const bf16* bg = bx + D;
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const uint4 ux = *reinterpret_cast<const uint4*>(bx + c * 8);
        const uint4 ug = *reinterpret_cast<const uint4*>(bg + c * 8);
        const float4 wa = *reinterpret_cast<const float4*>(sw + c * 8);
        const float4 wb = *reinterpret_cast<const float4*>(sw + c * 8 + 4);
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux.x, ux.y, ux.z, ux.w}, ag[4] = {ug.x, ug.y, ug.z, ug.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          m += fg.x * ws[2 * k] * fx.x + fg.y * ws[2 * k + 1] * fx.y;
        }
      }
    }
    m = warp_sum(m) / D;
    const float r3m = r * r * r * m;
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const uint4 ux = *reinterpret_cast<const uint4*>(bx + c * 8);
        const uint4 ug = *reinterpret_cast<const uint4*>(bg + c * 8);
        const float4 wa = *reinterpret_cast<const float4*>(sw + c * 8);
        const float4 wb = *reinterpret_cast<const float4*>(sw + c * 8 + 4);
        const float ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t ax[4] = {ux.x, ux.y, ux.z, ux.w}, ag[4] = {ug.x, ug.y, ug.z, ug.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fx = unpack_bf16(ax[k]), fg = unpack_bf16(ag[k]);
          o[k] = pack_bf16(r * fg.x * ws[2 * k] - fx.x * r3m, r * fg.y * ws[2 * k + 1] - fx.y * r3m);
          aw[j * 8 + 2 * k] += fg.x * fx.x * r;
          aw[j * 8 + 2 * k + 1] += fg.y * fx.y * r;
        }
        dr[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    buf ^= 1;
  }
  cp_async_wait_all();
  __syncthreads();
  // block sum of the warps' column partials: the staging area becomes [RB_NW][D] floats
  float* red = reinterpret_cast<float*>(stage);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      *reinterpret_cast<float4*>(red + (size_t)wid * D + c * 8) = make_float4(aw[j * 8], aw[j * 8 + 1], aw[j * 8 + 2], aw[j * 8 + 3]);
      *reinterpret_cast<float4*>(red + (size_t)wid * D + c * 8 + 4) =
          make_float4(aw[j * 8 + 4], aw[j * 8 + 5], aw[j * 8 + 6], aw[j * 8 + 7]);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < RB_NW; ++k) t += red[(size_t)k * D + c];
    part[(size_t)blockIdx.x * D + c] = t;
  }
}

// ---------------------------------------------------------------------------
// elementwise GELU / gate (vectorised by 8 bf16)
// ---------------------------------------------------------------------------
__global__ void gelu_fwd_k(const bf16* __restrict__ o, bf16* __restrict__ g, long n8) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    uint4 u = reinterpret_cast<const uint4*>(o)[i];
    uint32_t a[4] = {u.x, u.y, u.z, u.w}, r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16(a[k]);
      r[k] = pack_bf16(gelu_t(f.x), gelu_t(f.y));
    }
    reinterpret_cast<uint4*>(g)[i] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// out = x + g * sigmoid(h + b)      (x, out fp32; g, h bf16; b fp32 [D])
__global__ void glu_res_fwd_k(const float* __restrict__ x, const bf16* __restrict__ g,
                              const bf16* __restrict__ h, const float* __restrict__ b,
                              float* __restrict__ out, long n8, int D) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    uint4 ug = reinterpret_cast<const uint4*>(g)[i], uh = reinterpret_cast<const uint4*>(h)[i];
    uint32_t ag[4] = {ug.x, ug.y, ug.z, ug.w}, ah[4] = {uh.x, uh.y, uh.z, uh.w};
    float4 x0 = reinterpret_cast<const float4*>(x)[2 * i], x1 = reinterpret_cast<const float4*>(x)[2 * i + 1];
    float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w}, ov[8];
    int col = (int)((i * 8) % D);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 fg = unpack_bf16(ag[k]), fh = unpack_bf16(ah[k]);
      ov[2 * k] = xv[2 * k] + fg.x * sigmoidf_(fh.x + b[col + 2 * k]);
      ov[2 * k + 1] = xv[2 * k + 1] + fg.y * sigmoidf_(fh.y + b[col + 2 * k + 1]);
    }
    reinterpret_cast<float4*>(out)[2 * i] = make_float4(ov[0], ov[1], ov[2], ov[3]);
    reinterpret_cast<float4*>(out)[2 * i + 1] = make_float4(ov[4], ov[5], ov[6], ov[7]);
  }
}

// dh = dout * g * s(1-s) (bf16), dgp = dout * s (fp32); per-block partial rows of db.
template <int J>
__global__ void __launch_bounds__(CB_NT)
    glu_res_bwd_k(const float* __restrict__ dout, const bf16* __restrict__ g, const bf16* __restrict__ h,
                  const float* __restrict__ b, bf16* __restrict__ dh, float* __restrict__ dgp,
                  float* __restrict__ part, int T, int D) {
  extern __shared__ __align__(16) float red_smem[];   // [8][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* sb = red_smem + (size_t)wid * D;
  for (int c = lane * 4; c < D; c += 128) *reinterpret_cast<float4*>(sb + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  const int gw = blockIdx.x * (CB_NT / 32) + wid, nw = gridDim.x * (CB_NT / 32);
  for (int row = gw; row < T; row += nw) {
    const size_t o = (size_t)row * D;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * (lane + 32 * j);
      if (c < D) {
        const float4 gg = ld_bf16x4(g + o + c), hh = ld_bf16x4(h + o + c);
        const float4 bb = *reinterpret_cast<const float4*>(b + c);
        const float4 d = *reinterpret_cast<const float4*>(dout + o + c);
        const float sx = sigmoidf_(hh.x + bb.x), sy = sigmoidf_(hh.y + bb.y);
        const float sz = sigmoidf_(hh.z + bb.z), sw = sigmoidf_(hh.w + bb.w);
        const float4 v = make_float4(d.x * gg.x * sx * (1.f - sx), d.y * gg.y * sy * (1.f - sy),
                                     d.z * gg.z * sz * (1.f - sz), d.w * gg.w * sw * (1.f - sw));
        st_bf16x4(dh + o + c, v);
        *reinterpret_cast<float4*>(dgp + o + c) = make_float4(d.x * sx, d.y * sy, d.z * sz, d.w * sw);
        add4(sb + c, v);
      }
    }
  }
  __syncthreads();
  float* dst = part + (size_t)blockIdx.x * D;
  for (int c = threadIdx.x; c < D; c += CB_NT) {
    float t = 0.f;
    for (int k = 0; k < CB_NT / 32; ++k) t += red_smem[(size_t)k * D + c];
    dst[c] = t;
  }
}

// do = (dgp + dgm) * gelu'(o)  -> bf16
__global__ void gelu_bwd_k(const bf16* __restrict__ o, const float* __restrict__ dgp,
                           const bf16* __restrict__ dgm, bf16* __restrict__ dout, long n8) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    uint4 uo = reinterpret_cast<const uint4*>(o)[i], um = reinterpret_cast<const uint4*>(dgm)[i];
    uint32_t ao[4] = {uo.x, uo.y, uo.z, uo.w}, am[4] = {um.x, um.y, um.z, um.w}, r[4];
    float4 p0 = reinterpret_cast<const float4*>(dgp)[2 * i], p1 = reinterpret_cast<const float4*>(dgp)[2 * i + 1];
    float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 fo = unpack_bf16(ao[k]), fm = unpack_bf16(am[k]);
      r[k] = pack_bf16((pv[2 * k] + fm.x) * gelu_t_grad(fo.x), (pv[2 * k + 1] + fm.y) * gelu_t_grad(fo.y));
    }
    reinterpret_cast<uint4*>(dout)[i] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// ---------------------------------------------------------------------------
// Cross-entropy over bf16 logits (+ fp32 bias), one block per row.
// loss[row] = lse - logit[label]; logits <- w[row] * (softmax - onehot) in place.
// ---------------------------------------------------------------------------
__global__ void ce_fwd_bwd_k(bf16* __restrict__ logits, const float* __restrict__ bias,
                             const int64_t* __restrict__ labels, const float* __restrict__ wrow,
                             float* __restrict__ loss, int V, int ld) {
  int row = blockIdx.x;
  bf16* lr = logits + (size_t)row * ld;
  __shared__ float red[32];
  int tid = threadIdx.x, nt = blockDim.x;
  float mx = -INFINITY, se = 0.f;
  for (int c = tid; c < V; c += nt) {
    float v = __bfloat162float(lr[c]) + (bias ? bias[c] : 0.f);
    if (v > mx) { se = se * __expf(mx - v) + 1.f; mx = v; }
    else se += __expf(v - mx);
  }
  // block reduce of (mx, se)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, mx, o), s2 = __shfl_xor_sync(0xffffffffu, se, o);
    float m = fmaxf(mx, m2);
    se = (mx == -INFINITY ? 0.f : se * __expf(mx - m)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - m));
    mx = m;
  }
  __shared__ float smx[32], sse[32];
  int w = tid >> 5, lane = tid & 31;
  if (lane == 0) { smx[w] = mx; sse[w] = se; }
  __syncthreads();
  if (w == 0) {
    int nwarps = nt >> 5;
    mx = lane < nwarps ? smx[lane] : -INFINITY;
    se = lane < nwarps ? sse[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffffu, mx, o), s2 = __shfl_xor_sync(0xffffffffu, se, o);
      float m = fmaxf(mx, m2);
      se = (mx == -INFINITY ? 0.f : se * __expf(mx - m)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - m));
      mx = m;
    }
    if (lane == 0) { red[0] = mx; red[1] = logf(se); }
  }
  __syncthreads();
  float m = red[0], lse = m + red[1];
  int64_t lab = labels[row];
  float wr = wrow ? wrow[row] : 1.f;
  if (tid == 0) {
    float lv = __bfloat162float(lr[lab]) + (bias ? bias[lab] : 0.f);
    loss[row] = lse - lv;
  }
  __syncthreads();
  for (int c = tid; c < V; c += nt) {
    float v = __bfloat162float(lr[c]) + (bias ? bias[c] : 0.f);
    float p = __expf(v - lse);
    lr[c] = __float2bfloat16(wr * (p - (c == lab ? 1.f : 0.f)));
  }
}

// ---------------------------------------------------------------------------
// Optimizer: sum of squares, then fused clip + Adam(W) + bf16 copy.
// ---------------------------------------------------------------------------
__global__ void sumsq_k(const float* __restrict__ g, long n, float* __restrict__ out) {
  float s = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float v = g[i];
    s += v * v;
  }
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) atomicAdd(out, s);
  }
}

// One group: elements [0, n).  step is 1-based.  sumsq points at the global grad
// sum of squares; clip scale = max_norm / max(norm, max_norm) (optax clip_by_global_norm).
__global__ void adam_k(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                       float* __restrict__ v, bf16* __restrict__ pb, long n, const float* __restrict__ sumsq,
                       float max_norm, const float* __restrict__ lr_ptr, float b1, float b2, float eps,
                       float wd, float bc1, float bc2) {
  float scale = 1.f;
  if (sumsq && max_norm > 0.f) {
    float nrm = sqrtf(*sumsq);
    scale = nrm < max_norm ? 1.f : max_norm / nrm;
  }
  float lr = *lr_ptr;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float gi = g[i] * scale;
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float mh = mi / bc1, vh = vi / bc2;
    float pi = p[i];
    float upd = mh / (sqrtf(vh) + eps) + wd * pi;
    pi -= lr * upd;
    p[i] = pi;
    if (pb) pb[i] = __float2bfloat16(pi);
  }
}

}  // namespace ops
}  // namespace s0

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
using namespace s0::ops;

static int row_grid(long T, int sms) {
  long warps = T;
  long blocks = (warps * 32 + 255) / 256;
  long cap = (long)sms * 8;
  return (int)(blocks < cap ? blocks : cap);
}
template <typename K>
static void allow_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// grid for kernels that reduce columns: few blocks (2 per SM), each looping over rows
static int red_grid(long T, int sms) {
  long blocks = (T * 32 + 255) / 256;
  long cap = (long)sms * 6;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}
static int ew_grid(long n, int sms) {
  long blocks = (n + 255) / 256;
  long cap = (long)sms * 16;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

void ln_fwd_launch(const float* x, const float* w, const float* b, void* y, float* mean, float* rstd, long T,
                   int D, float eps, int sms, cudaStream_t st) {
  int gr = row_grid(T, sms);
  bf16* yp = reinterpret_cast<bf16*>(y);
  if (D <= 256) ln_fwd_k<8><<<gr, 256, 0, st>>>(x, w, b, yp, mean, rstd, (int)T, D, eps);
  else if (D <= 512) ln_fwd_k<16><<<gr, 256, 0, st>>>(x, w, b, yp, mean, rstd, (int)T, D, eps);
  else if (D <= 1024) ln_fwd_k<32><<<gr, 256, 0, st>>>(x, w, b, yp, mean, rstd, (int)T, D, eps);
  else ln_fwd_k<64><<<gr, 256, 0, st>>>(x, w, b, yp, mean, rstd, (int)T, D, eps);
}
int col_blocks(long T, int sms) {
  long b = (T + 15) / 16;
  long cap = 2L * sms;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}
static void col_sum(const float* part, int nblk, int sets, int D, float* o0, float* o1, cudaStream_t st) {
  int n = sets * D;
  col_sum_k<<<(n + 31) / 32, 256, 0, st>>>(part, nblk, sets, D, o0, o1);
}
void ln_bwd_launch(const void* dy, const float* x, const float* mean, const float* rstd, const float* w,
                   const float* dres, float* dx, float* dw, float* db, float* part, long T, int D, int sms,
                   cudaStream_t st) {
  const int gr = col_blocks(T, sms);
  const bf16* g = reinterpret_cast<const bf16*>(dy);
  const size_t sm = (size_t)(CB_NT / 32) * 2 * D * 4;
  if (D <= 256) { allow_smem(ln_bwd_k<2>, sm); ln_bwd_k<2><<<gr, CB_NT, sm, st>>>(g, x, mean, rstd, w, dres, dx, part, (int)T, D); }
  else if (D <= 512) { allow_smem(ln_bwd_k<4>, sm); ln_bwd_k<4><<<gr, CB_NT, sm, st>>>(g, x, mean, rstd, w, dres, dx, part, (int)T, D); }
  else if (D <= 1024) { allow_smem(ln_bwd_k<8>, sm); ln_bwd_k<8><<<gr, CB_NT, sm, st>>>(g, x, mean, rstd, w, dres, dx, part, (int)T, D); }
  else { allow_smem(ln_bwd_k<16>, sm); ln_bwd_k<16><<<gr, CB_NT, sm, st>>>(g, x, mean, rstd, w, dres, dx, part, (int)T, D); }
  col_sum(part, gr, 2, D, dw, db, st);
}
// pipelined variant (512 < D <= 1024): one block per SM; `part` holds >= sms rows of 2D
void ln_bwd_pipe_launch(const void* dy, const float* x, const float* mean, const float* rstd, const float* w,
                        const float* dres, float* dx, float* dw, float* db, float* part, long T, int D, int sms,
                        cudaStream_t st) {
  const int gr = (int)(T < sms ? T : sms);
  const size_t sm = sizeof(float) * ((size_t)3 * D + (size_t)LB_NW * 2 * (2 * D + D / 2));   // w, spare, stage
  allow_smem(ln_bwd_pipe_k, sm);
  ln_bwd_pipe_k<<<gr, LB_NW * 32, sm, st>>>(reinterpret_cast<const bf16*>(dy), x, mean, rstd, w, dres, dx, part,
                                            (int)T, D);
  col_sum(part, gr, 2, D, dw, db, st);
}
void rms_fwd_launch(const void* x, const float* w, void* y, float* rstd, long T, int D, float eps, int sms,
                    cudaStream_t st) {
  const int nv = D / 8, gr = row_grid(T, sms);
  const bf16* xp = reinterpret_cast<const bf16*>(x);
  bf16* yp = reinterpret_cast<bf16*>(y);
  if (nv <= 32) rms_fwd_k<1><<<gr, 256, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
  else if (nv <= 64) rms_fwd_k<2><<<gr, 256, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
  else if (nv <= 128) rms_fwd_k<4><<<gr, 256, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
  else rms_fwd_k<8><<<gr, 256, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
}
void rms_bwd_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                    float* part, long T, int D, int sms, cudaStream_t st) {
  const int gr = col_blocks(T, sms);
  const bf16* g = reinterpret_cast<const bf16*>(dy);
  const bf16* xp = reinterpret_cast<const bf16*>(x);
  bf16* o = reinterpret_cast<bf16*>(dx);
  const int nv = D / 8;
  const size_t sm = 8 * (size_t)D * 4;
  if (nv <= 32) { allow_smem(rms_bwd_k<1>, sm); rms_bwd_k<1><<<gr, 256, sm, st>>>(g, xp, w, rstd, o, part, (int)T, D); }
  else if (nv <= 64) { allow_smem(rms_bwd_k<2>, sm); rms_bwd_k<2><<<gr, 256, sm, st>>>(g, xp, w, rstd, o, part, (int)T, D); }
  else if (nv <= 128) { allow_smem(rms_bwd_k<4>, sm); rms_bwd_k<4><<<gr, 256, sm, st>>>(g, xp, w, rstd, o, part, (int)T, D); }
  else { allow_smem(rms_bwd_k<8>, sm); rms_bwd_k<8><<<gr, 256, sm, st>>>(g, xp, w, rstd, o, part, (int)T, D); }
  col_sum(part, gr, 1, D, dw, nullptr, st);
}
// wide rows (2048 < D <= 8192): one block per row; `part` holds >= rms_wide_blocks rows
int rms_wide_blocks(long T, int sms) {
  const long cap = 4L * sms;
  return (int)(T < cap ? (T > 0 ? T : 1) : cap);
}
void rms_fwd_wide_launch(const void* x, const float* w, void* y, float* rstd, long T, int D, float eps, int sms,
                         cudaStream_t st) {
  const long cap = 16L * sms;
  const int gr = (int)(T < cap ? (T > 0 ? T : 1) : cap);
  const bf16* xp = reinterpret_cast<const bf16*>(x);
  bf16* yp = reinterpret_cast<bf16*>(y);
  if (D <= RW_NT * 8 * 4) rms_fwd_wide_k<4><<<gr, RW_NT, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
  else rms_fwd_wide_k<8><<<gr, RW_NT, 0, st>>>(xp, w, yp, rstd, (int)T, D, eps);
}
void rms_bwd_wide_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                         float* part, long T, int D, int sms, cudaStream_t st) {
  const int gr = rms_wide_blocks(T, sms);
  const bf16* g = reinterpret_cast<const bf16*>(dy);
  const bf16* xp = reinterpret_cast<const bf16*>(x);
  bf16* o = reinterpret_cast<bf16*>(dx);
  if (D <= RW_NT * 8 * 4) rms_bwd_wide_k<4><<<gr, RW_NT, 0, st>>>(g, xp, w, rstd, o, part, (int)T, D);
  else rms_bwd_wide_k<8><<<gr, RW_NT, 0, st>>>(g, xp, w, rstd, o, part, (int)T, D);
  col_sum(part, gr, 1, D, dw, nullptr, st);
}
// pipelined variant for wide rows (D > 1024): one block per SM; `part` holds >= sms rows
void rms_bwd_pipe_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                         float* part, long T, int D, int sms, cudaStream_t st) {
  const int gr = (int)(T < sms ? T : sms);
  const size_t sm = (size_t)2 * D * 4 + (size_t)RB_NW * 4 * D * 2;
  allow_smem(rms_bwd_pipe_k<8>, sm);
  rms_bwd_pipe_k<8><<<gr, RB_NW * 32, sm, st>>>(reinterpret_cast<const bf16*>(dy), reinterpret_cast<const bf16*>(x),
                                                 w, rstd, reinterpret_cast<bf16*>(dx), part, (int)T, D);
  col_sum(part, gr, 1, D, dw, nullptr, st);
}
void gelu_fwd_launch(const void* o, void* g, long n, int sms, cudaStream_t st) {
  gelu_fwd_k<<<ew_grid(n / 8, sms), 256, 0, st>>>(reinterpret_cast<const bf16*>(o), reinterpret_cast<bf16*>(g),
                                                 n / 8);
}
void glu_res_fwd_launch(const float* x, const void* g, const void* h, const float* b, float* out, long n, int D,
                        int sms, cudaStream_t st) {
  glu_res_fwd_k<<<ew_grid(n / 8, sms), 256, 0, st>>>(x, reinterpret_cast<const bf16*>(g),
                                                    reinterpret_cast<const bf16*>(h), b, out, n / 8, D);
}
// grid of glu_res_bwd_k: four 8-warp blocks per SM (32 KB of shared memory each) keep more
// rows in flight than the two of col_blocks -- measured at 88,000 x 1024 on one B200:
// 290 us (2 per SM), 255 us (4), 267 us (6), 304 us (8)
int glu_bwd_blocks(long T, int sms) {
  long b = (T + 15) / 16;
  long cap = 4L * sms;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}
void glu_res_bwd_launch(const float* dout, const void* g, const void* h, const float* b, void* dh, float* dgp,
                        float* db, float* part, long T, int D, int sms, cudaStream_t st) {
  const int gr = glu_bwd_blocks(T, sms);
  const bf16* gp = reinterpret_cast<const bf16*>(g);
  const bf16* hp = reinterpret_cast<const bf16*>(h);
  bf16* dhp = reinterpret_cast<bf16*>(dh);
  const size_t sm = (size_t)(CB_NT / 32) * D * 4;
  if (D <= 256) { allow_smem(glu_res_bwd_k<2>, sm); glu_res_bwd_k<2><<<gr, CB_NT, sm, st>>>(dout, gp, hp, b, dhp, dgp, part, (int)T, D); }
  else if (D <= 512) { allow_smem(glu_res_bwd_k<4>, sm); glu_res_bwd_k<4><<<gr, CB_NT, sm, st>>>(dout, gp, hp, b, dhp, dgp, part, (int)T, D); }
  else if (D <= 1024) { allow_smem(glu_res_bwd_k<8>, sm); glu_res_bwd_k<8><<<gr, CB_NT, sm, st>>>(dout, gp, hp, b, dhp, dgp, part, (int)T, D); }
  else { allow_smem(glu_res_bwd_k<16>, sm); glu_res_bwd_k<16><<<gr, CB_NT, sm, st>>>(dout, gp, hp, b, dhp, dgp, part, (int)T, D); }
  col_sum(part, gr, 1, D, db, nullptr, st);
}
void gelu_bwd_launch(const void* o, const float* dgp, const void* dgm, void* dout, long n, int sms,
                     cudaStream_t st) {
  gelu_bwd_k<<<ew_grid(n / 8, sms), 256, 0, st>>>(reinterpret_cast<const bf16*>(o), dgp,
                                                 reinterpret_cast<const bf16*>(dgm), reinterpret_cast<bf16*>(dout),
                                                 n / 8);
}
void ce_launch(void* logits, const float* bias, const int64_t* labels, const float* wrow, float* loss, long T,
               int V, int ld, cudaStream_t st) {
  ce_fwd_bwd_k<<<(unsigned)T, 512, 0, st>>>(reinterpret_cast<bf16*>(logits), bias, labels, wrow, loss, V, ld);
}
void sumsq_launch(const float* g, long n, float* out, int sms, cudaStream_t st) {
  sumsq_k<<<ew_grid(n, sms), 256, 0, st>>>(g, n, out);
}
void adam_launch(float* p, const float* g, float* m, float* v, void* pb, long n, const float* sumsq,
                 float max_norm, const float* lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                 int sms, cudaStream_t st) {
  adam_k<<<ew_grid(n, sms), 256, 0, st>>>(p, g, m, v, reinterpret_cast<bf16*>(pb), n, sumsq, max_norm, lr, b1, b2,
                                         eps, wd, bc1, bc2);
}
