// tcgen05 / TMEM building blocks for sm_100a (inline PTX).
//
// Operand tiles live in shared memory in the K-major, 128-byte-swizzled layout:
// a tile of R rows x 64 bf16 (one 128-byte row per tile row), rows grouped in
// 8-row atoms of 1024 bytes, 16-byte chunk c of row r stored at chunk (c ^ (r & 7)).
// The tile base must be 1024-byte aligned.  A K=16 slice k of such a tile is
// addressed by advancing the descriptor's start address by 32*k bytes.
//
// The MMA is issued by one thread; completion is signalled through an mbarrier by
// tcgen05.commit; the accumulator (fp32) stays in tensor memory and is read back
// with tcgen05.ld (32 lanes x N columns per warp; warp w of a warpgroup owns lanes
// 32*(w%4) .. +31).  Every wait is bounded: on timeout the caller gets false and
// sets an error word instead of hanging.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace s0 {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of element (row r, k) inside a K-major SW128 tile of bf16 (k < 64)
__device__ __forceinline__ uint32_t sw128_off(int r, int k) {
  return (uint32_t)(r * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + ((k & 7) << 1));
}

// shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row atoms 1024 bytes apart
__device__ __forceinline__ uint64_t desc_sw128(const void* tile, int k_slice) {
  const uint32_t addr = smem_u32(tile) + 32u * (uint32_t)k_slice;
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);          // start address      [0,14)
  d |= (uint64_t)1 << 16;                            // leading byte offset [16,30) (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;                 // stride byte offset  [32,46): next 8-row atom
  d |= (uint64_t)1 << 46;                            // descriptor version 1 (sm100)
  d |= (uint64_t)2 << 61;                            // layout: SWIZZLE_128B
  return d;
}

// instruction descriptor, kind::f16: bf16 x bf16 -> fp32, both operands K-major
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate));
}

__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count) : "memory");
}

// bounded wait for the phase with parity `phase`; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t phase, long long max_polls = 1LL << 24) {
  const uint32_t a = smem_u32(mbar);
  for (long long i = 0; i < max_polls; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(a), "r"(phase)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// one arrival on an mbarrier (the phase completes when `count` arrivals are in)
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mbar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// one full warp: allocate `ncols` (power of two >= 32) TMEM columns; base address -> *slot
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 16 consecutive fp32 columns per warp (thread t <- lane t of the warp's quadrant)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace s0
