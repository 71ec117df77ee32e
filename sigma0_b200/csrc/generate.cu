// Per-token kernels of autoregressive message generation for sm_100a.
//
// gen_sample: syntax-masked sampling of the next token straight from the
//   decoder's fp32 logits (bias added here).  top_n == 1 is the argmax;
//   top_n == -1 samples the full softmax with the Gumbel-max trick
//   (argmax of logit + Gumbel noise has the softmax distribution; Gumbel, 1954;
//   Maddison et al., "A* Sampling", 2014).  This is the masked
//   fill_predicted_tok of the reference (src/base_model/inference/validation.py:217)
//   without materialising log-probabilities.  Uniforms come from a
//   counter-based hash (SplitMix64 finaliser; Steele, Lea and Flood,
//   "Fast splittable pseudorandom number generators", OOPSLA 2014) of
//   (seed, call counter, row, column), so a step replayed from a CUDA graph
//   draws fresh numbers when the device-side counter advances.
// gen_time_tokens: the time tokens of a message are computed, not sampled:
//   time = previous time + decoded delta_t, split into base-1000 digits
//   (_add_time_tokens, src/base_model/inference/generate.py:759).
#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace gen {

constexpr int NT = 512;

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(NT)
    gen_sample(const float* __restrict__ logits, int ldl, const float* __restrict__ bias,
               const unsigned char* __restrict__ allow, int V, unsigned long long seed,
               const long long* __restrict__ ctr, int salt, int top_n, int64_t* __restrict__ out, int out_stride) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* row = logits + (size_t)b * ldl;
  const unsigned long long base = mix64(seed ^ mix64(((unsigned long long)ctr[0] * 64ull + (unsigned long long)salt) * 0x100000001B3ull + b));
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = tid; v < V; v += NT) {
    if (!allow[v]) continue;
    float x = row[v] + (bias ? bias[v] : 0.f);
    if (top_n != 1) {
      unsigned long long z = mix64(base + (unsigned long long)v);
      float u = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
      x += -logf(-logf(u));
    }
    if (x > best || (x == best && v < bi)) { best = x; bi = v; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ob = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[NT / 32];
  __shared__ int si[NT / 32];
  if ((tid & 31) == 0) { sb[tid >> 5] = best; si[tid >> 5] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < NT / 32; ++w)
      if (sb[w] > best || (sb[w] == best && si[w] < bi)) { best = sb[w]; bi = si[w]; }
    out[(size_t)b * out_stride] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

// msg: [B, msg_len] int64 tokens of the message being generated; reads the
// delta-t tokens, writes the 5 absolute-time tokens, advances time [B, 2].
__global__ void gen_time_tokens(int64_t* __restrict__ msg, int msg_len, int dt_pos, int time_off,
                                int* __restrict__ time, int n) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  int64_t* m = msg + (size_t)b * msg_len;
  auto d = [&](int i) { return (int)m[dt_pos + i] - time_off; };
  const int dts = d(0);
  const int dtns = (d(1) * 1000 + d(2)) * 1000 + d(3);
  int ns = time[2 * b + 1] + dtns;
  const int extra = ns / 1000000000;
  ns -= extra * 1000000000;
  const int s = time[2 * b] + dts + extra;
  time[2 * b] = s;
  time[2 * b + 1] = ns;
  m[dt_pos + 4] = time_off + (s / 1000) % 1000;
  m[dt_pos + 5] = time_off + s % 1000;
  m[dt_pos + 6] = time_off + (ns / 1000000) % 1000;
  m[dt_pos + 7] = time_off + (ns / 1000) % 1000;
  m[dt_pos + 8] = time_off + ns % 1000;
}

}  // namespace gen
}  // namespace s0

void gen_sample_launch(const float* logits, int ldl, const float* bias, const unsigned char* allow, int V, int B,
                       unsigned long long seed, const long long* ctr, int salt, int top_n, int64_t* out,
                       int out_stride, cudaStream_t st) {
  s0::gen::gen_sample<<<B, s0::gen::NT, 0, st>>>(logits, ldl, bias, allow, V, seed, ctr, salt, top_n, out,
                                                  out_stride);
}

void gen_time_tokens_launch(int64_t* msg, int msg_len, int dt_pos, int time_off, int* time, int n,
                            cudaStream_t st) {
  s0::gen::gen_time_tokens<<<(n + 127) / 128, 128, 0, st>>>(msg, msg_len, dt_pos, time_off, time, n);
}
