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
// at most one of this thread's bulk stores may still be reading shared memory
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

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
           const __grid_constant__ CUtensorMap tmC) {
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
      constexpr int CW = OUT == 0 ? 64 : 32;            // output columns per 128-byte staged row
      // only chunks that are stored are staged: every staged chunk is followed by its store, so
      // the two buffers strictly alternate and "at most one store pending" protects the reuse
      const int cols_left = a.c_cols - w.tn * BN;
      const int c_end = row0 < a.c_rows ? (cols_left < BN ? cols_left : BN) : 0;
#pragma unroll 1
      for (int c = 0; c < c_end; c += CW, ++nb) {
        unsigned char* buf = epi + (size_t)(warp * 2 + (nb & 1)) * EPI_BUF;
        if (lane == 0) bulk_wait_read1();             // the store that used this buffer has read it
        __syncwarp();
        unsigned char* row = buf + lane * 128;
        if (OUT == 0) {
          float v[32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tc::tmem_ld32(tbase + (uint32_t)(c + 32 * h), v);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int chunk = 4 * h + q;
              *reinterpret_cast<uint4*>(row + (((chunk ^ (lane & 7)) & 7) << 4)) =
                  make_uint4(pack_bf16(v[8 * q + 0], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                             pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
            }
          }
        } else {
          float v[32];
          tc::tmem_ld32(tbase + (uint32_t)c, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row + (((q ^ (lane & 7)) & 7) << 4)) =
                make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        tc::fence_proxy_async();                      // generic-proxy writes -> the TMA store's reads
        __syncwarp();
        if (lane == 0) {                              // a box reaching past the output is clipped by TMA
          if (OUT == 2)
            tma_reduce_add_2d(&tmC, w.tn * BN + c, row0, buf);
          else
            tma_store_2d(&tmC, w.tn * BN + c, row0, buf);
          tc::bulk_commit();
        }
      }
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
  CUtensorMap tmA, tmB, tmC;
  const bool f32 = OUT != 0;
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
  auto* kern = gemm_k<AMN, BMN, OUT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
  const long units = (long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * a.split_k;
  const int grid = (int)(units < sms ? units : sms);
  kern<<<grid, NT, SMEM, st>>>(a, tmA, tmB, tmC);
  return (int)cudaGetLastError();
}
}  // namespace

int gemm_tc_launch(const GemmArgs& a, int sms, cudaStream_t st) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.split_k < 1) return -1;
  if (a.split_k > 1 && a.out_mode != 2) return -2;          // K splits sum through the reduce-add
  // TMA: 16-byte aligned bases, leading dimensions multiples of 16 bytes
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B) | reinterpret_cast<uintptr_t>(a.C)) % 16)
    return -3;
  const int ce = a.out_mode == 0 ? 2 : 4;
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16 || ((long)a.ldc * ce) % 16) return -4;
  if (a.c_rows < 1 || a.c_cols < 1 || a.c_rows > a.M || a.c_cols > a.N) return -5;
  const int key = (a.a_mn ? 4 : 0) | (a.b_mn ? 2 : 0);
#define S0_GEMM_CASE(AM, BMj, O)                             \
  if (key == ((AM ? 4 : 0) | (BMj ? 2 : 0)) && a.out_mode == O) \
    return launch_t<AM, BMj, O>(a, sms, st);
  S0_GEMM_CASE(false, true, 0)    // forward
  S0_GEMM_CASE(false, false, 0)   // input gradient
  S0_GEMM_CASE(true, true, 2)     // weight gradient, accumulated in fp32
  S0_GEMM_CASE(true, true, 1)     // weight gradient, stored in fp32
  S0_GEMM_CASE(false, true, 1)
  S0_GEMM_CASE(false, false, 1)
#undef S0_GEMM_CASE
  return -6;
}
