// Dense bf16 GEMM on the sm_100a tensor cores: C[M,N] (+)= A[M,K] . B[K,N], fp32 accumulation.
//
// The projections of the LOB models (Mamba3 in_proj / out_proj, the GLU gate, the decoder)
// and their two backward products run here instead of a library GEMM:
//
//   forward        y  = x . W          A = x  [M,K] K-major,      B = W  [K,N] MN-major
//   input grad     dx = dy . W^T       A = dy [M,K] K-major,      B = W  [N,K] K-major
//   weight grad    dW += x^T . dy      A = x  [K,M] MN-major,     B = dy [K,N] MN-major
//
// ("K-major": the operand's rows run along the reduction dimension in memory; "MN-major":
// its rows run along M or N.)  Both majors are read straight from the row-major tensors by
// TMA, so no operand is ever transposed in memory.
//
// One persistent CTA per SM (192 threads, warp-specialised):
//   warp 5   one thread streams 128 x 64 A and 256 x 64 B tiles with 2-D TMA loads (128-byte
//            swizzle, no multicast: every operand is this GPU's own memory) into a 4-stage
//            ring (full / empty mbarriers);
//   warp 4   one thread issues tcgen05.mma (M=128, N=256, K=16, bf16 -> fp32) into one of two
//            256-column tensor-memory accumulators, so a tile's products overlap the previous
//            tile's epilogue;
//   warps 0-3 read the accumulator back (tcgen05.ld, warp w owns rows 32w..32w+31), convert,
//            stage 32 x 128-byte blocks in swizzled shared memory (two per warp, alternating)
//            and write them with TMA: a bf16 or fp32 store, or an fp32 reduce-add -- the weight
//            gradient lands in the float32 gradient buffer with no separate widening pass and
//            accumulates across micro-batches (and across K splits).
// Edges need no special code: TMA zero-fills loads past M, N or K and clips stores.
// Work units are (output tile, K split) pairs dealt round robin; the K split (reduce-add only)
// keeps every SM busy when a long-K weight gradient has few output tiles.
// Waits are bounded: on timeout the kernel records a status word, stops issuing work, lets its
// copies land and returns.
#include <cuda.h>

#include "common.cuh"
#include "launchers.h"
#include "tc_common.cuh"
#include "tma_host.h"

namespace s0 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, NS = 4;
constexpr int NT = 192, EPI_WARPS = 4, MMA_WARP = 4, PROD_WARP = 5;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;   // 16 + 32 KB
constexpr int BOX = 64 * 128;                // one 64 x 64 bf16 SW128 box (MN-major pieces)
constexpr int EPI_BUF = 32 * 128;            // one warp's 32 rows x 128 bytes
constexpr size_t SMEM = 1024 + (size_t)NS * STAGE + (size_t)EPI_WARPS * 2 * EPI_BUF;
static_assert(SMEM <= 232448, "shared memory over the per-CTA limit");
constexpr uint32_t TMEM_COLS = 2 * BN;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(tc::smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(tc::smem_u32(src))
               : "memory");
}
// at most one / none of this thread's bulk stores may still be reading shared memory
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Output modes: 0 bf16 store, 1 fp32 store, 2 fp32 reduce-add, 3 the GLU block's fused
// epilogue: o = acc (bf16) and g = gelu(o) (bf16, through a second tensor map).
constexpr int OUT_BF16 = 0, OUT_F32 = 1, OUT_F32_ADD = 2, OUT_GELU = 3;

// One warp's share of an accumulator tile: rows row0..row0+31 (lane = row), columns
// col0 .. col0 + min(BN, c_cols - col0); staged 128 bytes per row in swizzled shared memory
// and written by TMA (partial boxes at the edges are clipped by the TMA unit).  Only chunks
// that are stored are staged, so the two staging buffers strictly alternate.
template <int OUT>
__device__ __forceinline__ void epilogue_rows(const GemmArgs& a, const CUtensorMap* tmC, const CUtensorMap* tmC2,
                                              unsigned char* mybuf, int lane, uint32_t tbase, int row0, int col0,
                                              int cbeg, int cspan, int& nb) {
  constexpr int CW = (OUT == OUT_F32 || OUT == OUT_F32_ADD) ? 32 : 64;   // output columns per 128-byte row
  const int cols_left = a.c_cols - col0;
  const int c_lim = cbeg + cspan < cols_left ? cbeg + cspan : cols_left;
  const int c_end = row0 < a.c_rows ? c_lim : 0;
#pragma unroll 1
  for (int c = cbeg; c < c_end; c += CW, ++nb) {
    unsigned char* buf = mybuf + (size_t)(nb & 1) * EPI_BUF;
    unsigned char* buf2 = mybuf + (size_t)((nb + 1) & 1) * EPI_BUF;
    if (lane == 0) {
      if (OUT == OUT_GELU)
        bulk_wait_read0();            // both buffers are written below
      else
        bulk_wait_read1();            // the store that used this buffer has read it
    }
    __syncwarp();
    unsigned char* rp = buf + lane * 128;
    unsigned char* rp2 = buf2 + lane * 128;
    if (OUT == OUT_F32 || OUT == OUT_F32_ADD) {
      float v[32];
      tc::tmem_ld32(tbase + (uint32_t)c, v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(rp + (((q ^ (lane & 7)) & 7) << 4)) =
            make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tc::tmem_ld32(tbase + (uint32_t)(c + 32 * h), v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = 4 * h + q;
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) w4[e] = pack_bf16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
          *reinterpret_cast<uint4*>(rp + (((chunk ^ (lane & 7)) & 7) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          if (OUT == OUT_GELU) {
            uint32_t g4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 ob = unpack_bf16(w4[e]);          // gelu of the stored (bf16) o
              g4[e] = pack_bf16(gelu_t(ob.x), gelu_t(ob.y));
            }
            *reinterpret_cast<uint4*>(rp2 + (((chunk ^ (lane & 7)) & 7) << 4)) =
                make_uint4(g4[0], g4[1], g4[2], g4[3]);
          }
        }
      }
    }
    tc::fence_proxy_async();          // generic-proxy writes -> the TMA store's reads
    __syncwarp();
    if (lane == 0) {
      if (OUT == OUT_F32_ADD)
        tma_reduce_add_2d(tmC, col0 + c, row0, buf);
      else
        tma_store_2d(tmC, col0 + c, row0, buf);
      if (OUT == OUT_GELU) tma_store_2d(tmC2, col0 + c, row0, buf2);
      tc::bulk_commit();
    }
  }
}

struct Unit {
  int tm, tn, kb0, kb1;
};
__device__ __forceinline__ Unit unit_of(const GemmArgs& a, long u, int tiles_n, int nkb) {
  const long t = u / a.split_k;
  const int s = (int)(u % a.split_k);
  Unit r;
  r.tm = (int)(t / tiles_n);
  r.tn = (int)(t % tiles_n);
  r.kb0 = (int)((long)s * nkb / a.split_k);
  r.kb1 = (int)((long)(s + 1) * nkb / a.split_k);
  return r;
}

// OUT: 0 = bf16 store, 1 = fp32 store, 2 = fp32 reduce-add
template <bool AMN, bool BMN, int OUT>
__global__ void __launch_bounds__(NT, 1)
    gemm_k(GemmArgs a, const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2];
  __shared__ uint32_t tslot;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  unsigned char* epi = base + (size_t)NS * STAGE;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) tc::tmem_alloc(&tslot, TMEM_COLS);
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&acc_full[i], 1);
      tc::mbar_init(&acc_empty[i], EPI_WARPS * 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tslot;
  const int tiles_m = (a.M + BM - 1) / BM, tiles_n = (a.N + BN - 1) / BN, nkb = (a.K + BK - 1) / BK;
  const long units = (long)tiles_m * tiles_n * a.split_k;
  bool ok = true;
  if (warp == PROD_WARP) {
    if (lane == 0) {
      long g = 0;
      for (long u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of(a, u, tiles_n, nkb);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++g) {
          const int s = (int)(g % NS);
          if (g >= NS && !tc::mbar_wait(&empty[s], (uint32_t)(((g / NS) - 1) & 1))) {
            ok = false;
            break;
          }
          unsigned char* sA = base + (size_t)s * STAGE;
          unsigned char* sB = sA + A_BYTES;
          tc::mbar_expect_tx(&full[s], STAGE);
          if (!AMN) {
            tma_load_2d(sA, &tmA, kb * BK, w.tm * BM, &full[s]);
          } else {
            tma_load_2d(sA, &tmA, w.tm * BM, kb * BK, &full[s]);
            tma_load_2d(sA + BOX, &tmA, w.tm * BM + 64, kb * BK, &full[s]);
          }
          if (!BMN) {
            tma_load_2d(sB, &tmB, kb * BK, w.tn * BN, &full[s]);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sB + c * BOX, &tmB, w.tn * BN + 64 * c, kb * BK, &full[s]);
          }
        }
      }
      // let every issued load land before the CTA can exit: the newest phase of each stage
      const long issued = g;
      for (long h = issued - NS > 0 ? issued - NS : 0; h < issued; ++h)
        tc::mbar_wait(&full[h % NS], (uint32_t)((h / NS) & 1));
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(BM, BN) | (AMN ? tc::IDESC_A_MN : 0u) | (BMN ? tc::IDESC_B_MN : 0u);
      long g = 0;
      int j = 0;
      for (long u = blockIdx.x; u < units && ok; u += gridDim.x, ++j) {
        const Unit w = unit_of(a, u, tiles_n, nkb);
        const int b = j & 1;
        if (j >= 2 && !tc::mbar_wait(&acc_empty[b], (uint32_t)(((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++g) {
          const int s = (int)(g % NS);
          if (!tc::mbar_wait(&full[s], (uint32_t)((g / NS) & 1))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          unsigned char* sA = base + (size_t)s * STAGE;
          unsigned char* sB = sA + A_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t ad = AMN ? tc::desc_mn_sw128(sA + ks * 2048, BOX) : tc::desc_sw128(sA, ks);
            const uint64_t bd = BMN ? tc::desc_mn_sw128(sB + ks * 2048, BOX) : tc::desc_sw128(sB, ks);
            tc::mma_bf16(acc, ad, bd, idesc, kb > w.kb0 || ks > 0);
          }
          tc::commit(&empty[s]);
        }
        if (!ok) break;
        tc::commit(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {
    // epilogue: warp w, lane l holds accumulator row 32w + l
    int j = 0, nb = 0;
    for (long u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      const Unit w = unit_of(a, u, tiles_n, nkb);
      const int b = j & 1;
      if (!tc::mbar_wait(&acc_full[b], (uint32_t)((j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int row0 = w.tm * BM + 32 * warp;
      const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(b * BN);
      epilogue_rows<OUT>(a, &tmC, &tmC2, epi + (size_t)warp * 2 * EPI_BUF, lane, tbase, row0, w.tn * BN, 0, BN, nb);
      tc::fence_before_sync();
      tc::mbar_arrive(&acc_empty[b]);                 // this thread's reads of accumulator b are done
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  if (!ok) atomicExch(a.status, 1);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}


// ---------------------------------------------------------------------------------------------
// Two-SM version: a cluster of 2 CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2.
// CTA r of the pair holds rows 128r..128r+127 of the A tile and columns 128r..128r+127 of the
// B tile in its own shared memory; the pair's leader (r = 0) issues M=256, N=256 MMAs that read
// both CTAs' halves, and each CTA's tensor memory receives its 128 rows of the product.  Per SM a
// 128 x 256 x 64 step stages 32 KB instead of 48 KB, which is what lets the tensor pipe outrun
// the L2.  Both CTAs' TMA loads complete on the leader's full barrier (the .cta_group::2 form of
// the load; no multicast qualifier anywhere), the leader's commits arrive on both CTAs' empty /
// accumulator-full barriers (CTA mask 0b11), and the peer's epilogue releases the accumulator
// with remote arrivals on the leader's barrier.
// ---------------------------------------------------------------------------------------------
// 7 warps: 0-3 epilogue (warp w reads TMEM lane quadrant w), 4 MMA issue (leader CTA only),
// 5 TMA loads, 6 the fused all-gather's copies (idle otherwise).  Six 32 KB stages: the pipeline depth is what the mainloop is sensitive to (five
// stages measured 2-5% slower; eight epilogue warps gained nothing).
constexpr int NS2 = 6;
constexpr int NT2 = 224, EPI_WARPS2 = 4, MMA_WARP2 = 4, PROD_WARP2 = 5, COPY_WARP2 = 6;
constexpr int H_BYTES = 128 * BK * 2;                          // one CTA's half of A or B per stage
constexpr int STAGE2 = 2 * H_BYTES;                            // 32 KB
constexpr size_t SMEM2 = 1024 + (size_t)NS2 * STAGE2 + (size_t)EPI_WARPS2 * 2 * EPI_BUF;
static_assert(SMEM2 <= 232448, "shared memory over the per-CTA limit");

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The copy warp of the fused all-gather (warp 6 of every CTA): this CTA's slice of every rank's
// row block of B, own block first, eight 16-byte loads in flight per lane; each block is counted
// once the slice has landed.
__device__ void ag_copy(const GemmArgs& a, int lane) {
  constexpr int nl = 32;
  bool ok = true;
  for (int i = 0; i < a.ag_world; ++i) {
    const int r = (a.ag_rank + i) % a.ag_world;
    if (r != a.ag_rank && ok) {
      long long it = 0;
      while (ld_acquire_sys(a.ag_ready[r]) < a.ag_seq) {
        if (++it > a.ag_spin) {
          ok = false;
          atomicExch(a.status, 3);            // a peer's shard never became current
          break;
        }
        __nanosleep(128);
      }
    }
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (ok) {
      const uint4* src = reinterpret_cast<const uint4*>(a.ag_src[r]);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.B)) +
                                            (size_t)r * a.ag_rows * a.ldb);
      const long n16 = (long)a.ag_rows * a.ldb / 8;
      const long per = (n16 + gridDim.x - 1) / gridDim.x;
      const long lo = (long)blockIdx.x * per, hi = lo + per < n16 ? lo + per : n16;
      long j = lo + lane;
      for (; j + 7 * nl < hi; j += 8 * nl) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = src[j + k * nl];
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[j + k * nl] = v[k];
      }
      for (; j < hi; j += nl) dst[j] = src[j];
    }
    __threadfence();                            // the slice is visible GPU-wide before it is counted
    __syncwarp();
    if (lane == 0) atomicAdd(a.ag_count + r, 1);   // counted even after a timeout: nobody waits forever
  }
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(tc::smem_u32(p)), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory completing on the pair leader's mbarrier
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t mbar_cl) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cl)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)acc));
}
// arrive once on the barrier at this offset in both CTAs of the pair when the leader's MMAs finish
__device__ __forceinline__ void commit_pair(uint64_t* mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          tc::smem_u32(mbar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t mbar_cl) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mbar_cl) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <bool AMN, bool BMN, int OUT>
__global__ void __launch_bounds__(NT2, 1)
    gemm2_k(GemmArgs a, const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[NS2], empty[NS2], acc_full[2], acc_empty[2];
  __shared__ uint32_t tslot;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  unsigned char* epi = base + (size_t)NS2 * STAGE2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();              // 0 = the pair's leader
  const bool leader = rank == 0;
  if (warp == 0) tmem_alloc_pair(&tslot, TMEM_COLS);
  if (tid == 0) {
    for (int i = 0; i < NS2; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&acc_full[i], 1);
      tc::mbar_init(&acc_empty[i], 2 * EPI_WARPS2 * 32); // both CTAs' epilogue threads
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc::fence_before_sync();
  cluster_sync();                                     // both CTAs' barriers exist before any remote use
  tc::fence_after_sync();
  const uint32_t tmem = tslot;
  const int tiles_m = (a.M + 255) / 256, tiles_n = (a.N + 255) / 256, nkb = (a.K + BK - 1) / BK;
  const long units = (long)tiles_m * tiles_n * a.split_k;
  const long pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  bool ok = true;
  if (warp == COPY_WARP2) {
    if (a.ag_world > 1) ag_copy(a, lane);
  } else if (warp == PROD_WARP2) {
    const bool ag = a.ag_world > 1;
    if (lane == 0) {
      // fused all-gather: k-blocks start at this rank's own row block (copied locally first);
      // a block of another rank is loaded once every CTA has copied its slice of it
      const int kb_rot = ag ? a.ag_rank * (a.ag_rows / BK) : 0;
      uint32_t ready = 0;
      long g = 0;
      for (long u = pair; u < units && ok; u += npairs) {
        const long t = u / a.split_k;
        const int sk = (int)(u % a.split_k);
        const int tm = (int)(t / tiles_n), tn = (int)(t % tiles_n);
        const int kb0 = (int)((long)sk * nkb / a.split_k), kb1 = (int)((long)(sk + 1) * nkb / a.split_k);
        const int ra = tm * 256 + 128 * (int)rank, rb = tn * 256 + 128 * (int)rank;
        for (int kbi = kb0; kbi < kb1; ++kbi, ++g) {
          const int kb = ag ? (kbi + kb_rot) % nkb : kbi;
          const int s = (int)(g % NS2);
          if (g >= NS2 && !tc::mbar_wait(&empty[s], (uint32_t)(((g / NS2) - 1) & 1))) {
            ok = false;
            break;
          }
          if (ag) {
            const int owner = kb * BK / a.ag_rows;
            if (!(ready >> owner & 1u)) {
              long long it = 0;
              while (ld_acquire_gpu(a.ag_count + owner) < (int)gridDim.x) {
                if (++it > a.ag_spin) {
                  ok = false;
                  break;
                }
                __nanosleep(64);
              }
              if (!ok) break;
              // generic-proxy stores (the copy lanes of every CTA) -> this thread's TMA reads
              asm volatile("fence.proxy.async.global;" ::: "memory");
              ready |= 1u << owner;
            }
          }
          unsigned char* sA = base + (size_t)s * STAGE2;
          unsigned char* sB = sA + H_BYTES;
          const uint32_t fb = map_to_rank(&full[s], 0);
          if (leader) tc::mbar_expect_tx(&full[s], 2 * STAGE2);   // both CTAs' halves
          if (!AMN) {
            tma_load_2d_pair(sA, &tmA, kb * BK, ra, fb);
          } else {
            tma_load_2d_pair(sA, &tmA, ra, kb * BK, fb);
            tma_load_2d_pair(sA + BOX, &tmA, ra + 64, kb * BK, fb);
          }
          if (!BMN) {
            tma_load_2d_pair(sB, &tmB, kb * BK, rb, fb);
          } else {
            tma_load_2d_pair(sB, &tmB, rb, kb * BK, fb);
            tma_load_2d_pair(sB + BOX, &tmB, rb + 64, kb * BK, fb);
          }
        }
      }
      // every issued load has landed once the MMAs that read it have committed: wait for the
      // newest phase of each stage's empty barrier (bounded)
      for (long h = g - NS2 > 0 ? g - NS2 : 0; h < g; ++h) tc::mbar_wait(&empty[h % NS2], (uint32_t)((h / NS2) & 1));
    }
    __syncwarp();
  } else if (warp == MMA_WARP2) {
    if (leader && lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(256, 256) | (AMN ? tc::IDESC_A_MN : 0u) | (BMN ? tc::IDESC_B_MN : 0u);
      long g = 0;
      int j = 0;
      for (long u = pair; u < units && ok; u += npairs, ++j) {
        const long t = u / a.split_k;
        const int sk = (int)(u % a.split_k);
        const int kb0 = (int)((long)sk * nkb / a.split_k), kb1 = (int)((long)(sk + 1) * nkb / a.split_k);
        (void)t;
        const int b = j & 1;
        if (j >= 2 && !tc::mbar_wait(&acc_empty[b], (uint32_t)(((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = (int)(g % NS2);
          if (!tc::mbar_wait(&full[s], (uint32_t)((g / NS2) & 1))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          unsigned char* sA = base + (size_t)s * STAGE2;
          unsigned char* sB = sA + H_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t ad = AMN ? tc::desc_mn_sw128(sA + ks * 2048, BOX) : tc::desc_sw128(sA, ks);
            const uint64_t bd = BMN ? tc::desc_mn_sw128(sB + ks * 2048, BOX) : tc::desc_sw128(sB, ks);
            mma_pair(acc, ad, bd, idesc, kb > kb0 || ks > 0);
          }
          commit_pair(&empty[s]);
        }
        if (!ok) break;
        commit_pair(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {
    // epilogue: CTA r, warp w, lane l holds row 128r + 32w + l of the 256-row tile
    const uint32_t acc_empty_cl0 = map_to_rank(&acc_empty[0], 0), acc_empty_cl1 = map_to_rank(&acc_empty[1], 0);
    int j = 0, nb = 0;
    for (long u = pair; u < units; u += npairs, ++j) {
      const long t = u / a.split_k;
      const int tm = (int)(t / tiles_n), tn = (int)(t % tiles_n);
      const int b = j & 1;
      if (!tc::mbar_wait(&acc_full[b], (uint32_t)((j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int row0 = tm * 256 + 128 * (int)rank + 32 * warp;
      const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(b * BN);
      epilogue_rows<OUT>(a, &tmC, &tmC2, epi + (size_t)warp * 2 * EPI_BUF, lane, tbase, row0, tn * BN, 0, BN, nb);
      tc::fence_before_sync();
      if (leader)
        tc::mbar_arrive(&acc_empty[b]);
      else
        arrive_remote(b ? acc_empty_cl1 : acc_empty_cl0);   // the leader's MMA warp waits for both CTAs
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  if (!ok) atomicExch(a.status, 1);
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();                                       // the leader's MMAs may read this CTA's smem until here
  if (warp == 0) tmem_dealloc_pair(tmem, TMEM_COLS);
}

}  // namespace gemm
}  // namespace s0

namespace {
using s0::gemm::BK;
using s0::gemm::BM;
using s0::gemm::BN;

// 2-D bf16/fp32 tensor map over a row-major [rows, cols] matrix with leading dimension ld
// (elements), box box_cols x box_rows, 128-byte swizzle
int encode_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, long rows, long cols, long ld,
              int box_cols, int box_rows) {
  const auto enc = s0::tensor_map_encoder();
  if (!enc) return -10;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * esize};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
                 CUDA_SUCCESS
             ? 0
             : -11;
}

template <bool AMN, bool BMN, int OUT>
int launch_t(const GemmArgs& a, int sms, cudaStream_t st) {
  using namespace s0::gemm;
  CUtensorMap tmA, tmB, tmC, tmC2;
  const bool f32 = OUT == 1 || OUT == 2;
  // A: K-major [M, K] (box 64 K x 128 rows) or MN-major [K, M] (box 64 M x 64 K)
  int e = AMN ? encode_2d(&tmA, a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, a.lda, 64, 64)
              : encode_2d(&tmA, a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, 64, BM);
  if (e) return e;
  // B: K-major [N, K] (box 64 K x 256 rows) or MN-major [K, N] (box 64 N x 64 K)
  e = BMN ? encode_2d(&tmB, a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.N, a.ldb, 64, 64)
          : encode_2d(&tmB, a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, 64, BN);
  if (e) return e;
  // C: [c_rows, c_cols] with leading dimension ldc; box = one warp's 32 rows x 128 bytes
  e = encode_2d(&tmC, a.C, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, f32 ? 4 : 2,
                a.c_rows, a.c_cols, a.ldc, f32 ? 32 : 64, 32);
  if (e) return e;
  tmC2 = tmC;
  if (OUT == 3 && (e = encode_2d(&tmC2, a.C2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.c_rows, a.c_cols, a.ldc2, 64, 32)))
    return e;
  auto* kern = gemm_k<AMN, BMN, OUT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
  const long units = (long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * a.split_k;
  const int grid = (int)(units < sms ? units : sms);
  kern<<<grid, NT, SMEM, st>>>(a, tmA, tmB, tmC, tmC2);
  return (int)cudaGetLastError();
}
template <bool AMN, bool BMN, int OUT>
int launch_pair(const GemmArgs& a, int sms, cudaStream_t st) {
  using namespace s0::gemm;
  CUtensorMap tmA, tmB, tmC, tmC2;
  const bool f32 = OUT == 1 || OUT == 2;
  // each CTA loads a 128-row (K-major) or 2 x 64-column (MN-major) half of the A and B tiles
  int e = AMN ? encode_2d(&tmA, a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, a.lda, 64, 64)
              : encode_2d(&tmA, a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, 64, 128);
  if (e) return e;
  e = BMN ? encode_2d(&tmB, a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.N, a.ldb, 64, 64)
          : encode_2d(&tmB, a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, 64, 128);
  if (e) return e;
  e = encode_2d(&tmC, a.C, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, f32 ? 4 : 2,
                a.c_rows, a.c_cols, a.ldc, f32 ? 32 : 64, 32);
  if (e) return e;
  tmC2 = tmC;
  if (OUT == 3 && (e = encode_2d(&tmC2, a.C2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.c_rows, a.c_cols, a.ldc2, 64, 32)))
    return e;
  auto* kern = gemm2_k<AMN, BMN, OUT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM2);
  const long units = (long)((a.M + 255) / 256) * ((a.N + 255) / 256) * a.split_k;
  long pairs = units < sms / 2 ? units : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(NT2);
  cfg.dynamicSmemBytes = SMEM2;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent pairs must all be resident at once (a pair lives in one GPC): no more pairs than
  // the device can hold together
  int max_clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&max_clusters, (const void*)kern, &cfg) == cudaSuccess && max_clusters > 0 &&
      pairs > max_clusters)
    pairs = max_clusters;
  if (pairs < 1) return -7;
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, a, tmA, tmB, tmC, tmC2);
  return err == cudaSuccess ? 0 : (int)err;
}
}  // namespace

// 1: the two-SM kernel (default), 0: the one-SM kernel
int g_gemm_pair = 1;
void gemm_tc_set_pair(int on) { g_gemm_pair = on; }

// K split for a reduce-add product: the split (1..16, at least 16 K-blocks per part) whose work
// units fill the last wave of `slots` persistent workers best
static int pick_split(long tiles, int K, int slots) {
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 16; ++s) {
    if (s > 1 && (K + BK - 1) / BK / s < 16) break;
    const long units = tiles * s, waves = (units + slots - 1) / slots;
    const double eff = (double)units / (double)(waves * slots);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

int gemm_tc_launch(const GemmArgs& a_in, int sms, cudaStream_t st) {
  GemmArgs a = a_in;
  if (a.split_k == 0) {        // auto: only for the reduce-add mode
    if (a.out_mode != 2) {
      a.split_k = 1;
    } else if (g_gemm_pair) {
      a.split_k = pick_split((long)((a.M + 255) / 256) * ((a.N + 255) / 256), a.K, sms / 2);
    } else {
      a.split_k = pick_split((long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN), a.K, sms);
    }
  }
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.split_k < 1) return -1;
  if (a.split_k > 1 && a.out_mode != 2) return -2;          // K splits sum through the reduce-add
  // TMA: 16-byte aligned bases, leading dimensions multiples of 16 bytes
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B) | reinterpret_cast<uintptr_t>(a.C)) % 16)
    return -3;
  const int ce = (a.out_mode == 1 || a.out_mode == 2) ? 4 : 2;
  if (a.ag_world > 1) {       // fused all-gather: two-SM kernel, MN-major B rows split in 64-row blocks
    if (!g_gemm_pair || a.a_mn || !a.b_mn || a.split_k != 1 || a.ag_world > 8 || a.ag_rows % BK ||
        (long)a.ag_rows * a.ag_world != a.K || a.ldb != a.N || a.ag_count == nullptr)
      return -10;
    for (int r = 0; r < a.ag_world; ++r)
      if (reinterpret_cast<uintptr_t>(a.ag_src[r]) % 16 || a.ag_ready[r] == nullptr) return -11;
  }
  if (a.out_mode == 3) {      // fused epilogue: whole 64-column chunks, an aligned second output
    if (a.c_cols % 64) return -8;
    if (a.out_mode == 3 && (reinterpret_cast<uintptr_t>(a.C2) % 16 || (a.ldc2 * 2) % 16)) return -9;
  }
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16 || ((long)a.ldc * ce) % 16) return -4;
  if (a.c_rows < 1 || a.c_cols < 1 || a.c_rows > a.M || a.c_cols > a.N) return -5;
  const int key = (a.a_mn ? 4 : 0) | (a.b_mn ? 2 : 0);
#define S0_GEMM_CASE(AM, BMj, O)                                                                   \
  if (key == ((AM ? 4 : 0) | (BMj ? 2 : 0)) && a.out_mode == O)                                       \
    return g_gemm_pair ? launch_pair<AM, BMj, O>(a, sms, st) : launch_t<AM, BMj, O>(a, sms, st);
  S0_GEMM_CASE(false, true, 0)    // forward
  S0_GEMM_CASE(false, false, 0)   // input gradient
  S0_GEMM_CASE(true, true, 2)     // weight gradient, accumulated in fp32
  S0_GEMM_CASE(true, true, 1)     // weight gradient, stored in fp32
  S0_GEMM_CASE(false, true, 1)
  S0_GEMM_CASE(false, false, 1)
  S0_GEMM_CASE(false, true, 3)    // o = x . W and g = gelu(o)
#undef S0_GEMM_CASE
  return -6;
}
