// Embedding gathers for the message encoders (sm_100a): the token embedding of the LOB model
// and the 1-token model's FieldEmbedding -- the sum over the 24 fields of each field's own
// table row (src/base_model/models/lob_seq_model.py:370, :1071-1087).
//
// Forward: one warp per token; the warp adds the rows of its token's fields, float4 lanes
// over the model width (fp32 tables, fp32 output).  Backward: the same walk scatter-adds the
// output gradient into each table's gradient with vector fp32 atomics (red.global.add.v4).
// Indices outside a table are clamped to its last row, as an XLA gather clamps.
#include <cuda_runtime.h>

#include "launchers.h"

namespace {

constexpr int NT = 256;

__device__ __forceinline__ int clamp_row(long long v, int rows) {
  return v < 0 ? 0 : (v >= rows ? rows - 1 : (int)v);
}

__global__ void __launch_bounds__(NT) embed_sum_fwd_k(EmbedSumArgs a) {
  const long long t = ((long long)blockIdx.x * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const int nv = a.D / 4;
  const long long* id = a.idx + t * a.nf;
  float4* out = reinterpret_cast<float4*>(a.out + t * a.D);
  for (int c0 = 0; c0 < nv; c0 += 32 * 4) {
    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int f = 0; f < a.nf; ++f) {
      const int row = clamp_row(id[f], a.rows[f]);
      const float4* src = reinterpret_cast<const float4*>(a.tab[f] + (size_t)row * a.D);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = c0 + k * 32 + lane;
        if (c < nv) {
          const float4 v = __ldg(src + c);
          acc[k].x += v.x; acc[k].y += v.y; acc[k].z += v.z; acc[k].w += v.w;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + k * 32 + lane;
      if (c < nv) out[c] = acc[k];
    }
  }
}

__global__ void __launch_bounds__(NT) embed_sum_bwd_k(EmbedSumBwdArgs a) {
  const long long t = ((long long)blockIdx.x * NT + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const int nv = a.D / 4;
  const long long* id = a.idx + t * a.nf;
  const float4* g = reinterpret_cast<const float4*>(a.dout + t * a.D);
  for (int f = 0; f < a.nf; ++f) {
    const int row = clamp_row(id[f], a.rows[f]);
    float4* dst = reinterpret_cast<float4*>(a.gtab[f] + (size_t)row * a.D);
    for (int c = lane; c < nv; c += 32) atomicAdd(dst + c, __ldg(g + c));
  }
}

}  // namespace

int embed_sum_fwd_launch(const EmbedSumArgs& a, cudaStream_t st) {
  if (a.T <= 0) return 0;
  if (a.nf <= 0 || a.nf > EMBED_MAX_FIELDS || a.D % 4) return -1;
  const long long blocks = (a.T * 32 + NT - 1) / NT;
  embed_sum_fwd_k<<<(unsigned)blocks, NT, 0, st>>>(a);
  return (int)cudaGetLastError();
}

int embed_sum_bwd_launch(const EmbedSumBwdArgs& a, cudaStream_t st) {
  if (a.T <= 0) return 0;
  if (a.nf <= 0 || a.nf > EMBED_MAX_FIELDS || a.D % 4) return -1;
  const long long blocks = (a.T * 32 + NT - 1) / NT;
  embed_sum_bwd_k<<<(unsigned)blocks, NT, 0, st>>>(a);
  return (int)cudaGetLastError();
}
