// Self-test of the tcgen05 building blocks (tc_common.cuh): one CTA computes
// D = A . B^T for A (M x K) and B (N x K) bf16 with K-major swizzled operands in
// shared memory, the accumulator in tensor memory.  Used by the GPU tests to pin
// the descriptor encodings and the TMEM row layout before kernels rely on them.
#include "tc_common.cuh"
#include "launchers.h"

namespace s0 {
namespace tct {

using bf16 = __nv_bfloat16;

__global__ void __launch_bounds__(128) tc_gemm_test_k(const bf16* __restrict__ A, const bf16* __restrict__ B,
                                                      float* __restrict__ D, int M, int N, int K,
                                                      int* __restrict__ err) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t mbar;
  __shared__ uint32_t tslot;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = K / 64;
  unsigned char* sA = base;
  unsigned char* sB = base + (size_t)nk * M * 128;
  if (warp == 0) tc::tmem_alloc(&tslot, 128);
  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < M * K; i += 128) {
    const int r = i / K, k = i % K;
    *reinterpret_cast<bf16*>(sA + (size_t)(k / 64) * M * 128 + tc::sw128_off(r, k % 64)) = A[i];
  }
  for (int i = tid; i < N * K; i += 128) {
    const int r = i / K, k = i % K;
    *reinterpret_cast<bf16*>(sB + (size_t)(k / 64) * N * 128 + tc::sw128_off(r, k % 64)) = B[i];
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tslot;
  if (tid == 0) {
    const uint32_t id = tc::idesc_bf16(M, N);
    for (int kt = 0; kt < nk; ++kt)
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem, tc::desc_sw128(sA + (size_t)kt * M * 128, ks), tc::desc_sw128(sB + (size_t)kt * N * 128, ks),
                     id, (kt | ks) != 0);
    tc::commit(&mbar);
  }
  const bool ok = tc::mbar_wait(&mbar, 0);
  if (!ok && lane == 0) atomicExch(err, 1);
  tc::fence_after_sync();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      tc::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
      const int row = 32 * warp + lane;
#pragma unroll
      for (int j = 0; j < 16; ++j) D[(size_t)row * N + c0 + j] = v[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 128);
}

}  // namespace tct
}  // namespace s0

int tc_gemm_test_launch(const void* A, const void* B, float* D, int M, int N, int K, int* err, cudaStream_t st) {
  if (!((M == 64 || M == 128) && (N == 64 || N == 128) && (K == 64 || K == 128))) return -1;
  const size_t smem = 1024 + (size_t)(K / 64) * (M + N) * 128;
  cudaFuncSetAttribute(s0::tct::tc_gemm_test_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  s0::tct::tc_gemm_test_k<<<1, 128, smem, st>>>(reinterpret_cast<const __nv_bfloat16*>(A),
                                                 reinterpret_cast<const __nv_bfloat16*>(B), D, M, N, K, err);
  return 0;
}
