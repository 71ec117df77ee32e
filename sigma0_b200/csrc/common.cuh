// Shared device helpers for the sm_100a kernels of sigma0_b200.
//
// Warp-level bf16 tensor-core tiles (ldmatrix + mma.m16n8k16), cp.async tile
// copies, and small math helpers.  The fragment conventions used throughout:
//   A (16x16, row-major):  a0=(g, 2t..2t+1) a1=(g+8, 2t..) a2=(g, 8+2t..) a3=(g+8, 8+2t..)
//   B (16x8):             b0=(k 2t..2t+1, n g) b1=(k 8+2t.., n g)
//   C/D (16x8, f32):      c0,c1=(g, 2t..2t+1) c2,c3=(g+8, 2t..2t+1)
// with g = lane/4 and t = lane%4.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define S0_DEV __device__ __forceinline__

namespace s0 {

S0_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async copy global->shared; src_bytes < 16 zero-fills the rest.
S0_DEV void cp_async16(void* smem, const void* gmem, int src_bytes = 16) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes));
}
S0_DEV void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
S0_DEV void cp_async4(void* smem, const void* gmem, int src_bytes = 4) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes));
}
S0_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
S0_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }
// wait until at most N of the most recently committed groups are still in flight
template <int N>
S0_DEV void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

S0_DEV void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
S0_DEV void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

S0_DEV void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

S0_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
S0_DEV float2 unpack_bf16(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// ---------------------------------------------------------------------------
// Warp tile loaders over row-major bf16 smem matrices with leading dim `ld`.
// ---------------------------------------------------------------------------

// A fragment for rows [m0,m0+16) x k [k0,k0+16) of a matrix stored A[m][k].
S0_DEV void load_a(uint32_t* a, const __nv_bfloat16* s, int ld, int m0, int k0, int lane) {
  int r = m0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  int c = k0 + (lane >> 4) * 8;
  ldsm_x4(a[0], a[1], a[2], a[3], s + r * ld + c);
}
// A fragment when the matrix is stored transposed, At[k][m] (A[m][k] = At[k][m]).
S0_DEV void load_a_t(uint32_t* a, const __nv_bfloat16* s, int ld, int m0, int k0, int lane) {
  int j = lane >> 3;
  int r = k0 + (lane & 7) + (j >> 1) * 8;
  int c = m0 + (j & 1) * 8;
  ldsm_x4_t(a[0], a[1], a[2], a[3], s + r * ld + c);
}
// B fragments for two n-tiles [n0,n0+16) x k [k0,k0+16), matrix stored Bt[n][k].
// b[0],b[1] -> n-tile n0; b[2],b[3] -> n-tile n0+8.
S0_DEV void load_b_nk(uint32_t* b, const __nv_bfloat16* s, int ld, int n0, int k0, int lane) {
  int j = lane >> 3;
  int r = n0 + (lane & 7) + (j >> 1) * 8;
  int c = k0 + (j & 1) * 8;
  ldsm_x4(b[0], b[1], b[2], b[3], s + r * ld + c);
}
// Same fragments when the matrix is stored B[k][n] (n contiguous).
S0_DEV void load_b_kn(uint32_t* b, const __nv_bfloat16* s, int ld, int n0, int k0, int lane) {
  int j = lane >> 3;
  int r = k0 + (lane & 7) + (j & 1) * 8;
  int c = n0 + (j >> 1) * 8;
  ldsm_x4_t(b[0], b[1], b[2], b[3], s + r * ld + c);
}

// Accumulator n-tiles (2*kk, 2*kk+1) of a 16-row f32 tile -> bf16 A fragment for k-step kk.
S0_DEV void acc_to_a(uint32_t* a, const float* c0, const float* c1) {
  a[0] = pack_bf16(c0[0], c0[1]);
  a[1] = pack_bf16(c0[2], c0[3]);
  a[2] = pack_bf16(c1[0], c1[1]);
  a[3] = pack_bf16(c1[2], c1[3]);
}

// fast division (__fdividef): the IEEE-exact division is a multi-instruction sequence and
// the logistic's operand is >= 1, where the fast form is within 2 ulp (and gives 0 for
// an infinite exponential)
S0_DEV float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
S0_DEV float softplusf_(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

S0_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// tanh-approximated GELU (flax's approximate gelu) and its derivative
constexpr float K_GELU = 0.7978845608028654f;   // sqrt(2/pi)
constexpr float C_GELU = 0.044715f;
S0_DEV float gelu_t(float x) {
  float u = K_GELU * (x + C_GELU * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}
S0_DEV float gelu_t_grad(float x) {
  float u = K_GELU * (x + C_GELU * x * x * x);
  float th = tanhf(u);
  return 0.5f * (1.f + th) + 0.5f * x * (1.f - th * th) * K_GELU * (1.f + 3.f * C_GELU * x * x);
}

}  // namespace s0
