// Tensor-parallel row-parallel projection fused with its all-reduce, for sm_100a.
//
// out = sum_r A_r . W_r over the ranks r of a tensor-parallel group, where rank r
// holds A_r [M, K] (its heads' activations) and W_r [K, N] (its rows of the
// projection, passed transposed as Bt_r [N, K]).  This replaces "GEMM, then NCCL
// all-reduce" (the psum after the reference's row-parallel out_proj,
// src/base_model/models/mamba3.py:209-233) with ONE cooperative kernel per rank:
//
//   phase 1  persistent loop over 128 x BN output tiles (BN = 256 when the width
//            allows, else 128), warp-specialised: one thread streams the
//            operands with TMA (tiled, 128-byte swizzle, no multicast: the
//            operands are this GPU's own memory) into K-major stages (full /
//            empty mbarriers), one thread issues tcgen05.mma into one of two
//            tensor-memory accumulators (the next tile's products overlap the
//            previous tile's epilogue), four epilogue warps read the tile back
//            with tcgen05.ld, stage 64 columns of their rows as bf16 in shared
//            memory and store whole 128-byte row segments into this rank's slot
//            of the receive buffer of the rank that owns the tile's rows (row
//            tiles are dealt round robin) -- peer memory over NVLink, so the
//            reduce-scatter overlaps the remaining tiles;
//   phase 2  cross-rank barrier (flags in peer memory, bounded spins);
//   phase 3  every rank bulk-copies row blocks of its own receive slots into shared
//            memory (a 3-stage ring), sums the world partials in fp32, rounds to
//            bf16 and stores the rows into every rank's output buffer (peer
//            stores: the all-gather);
//   phase 4  cross-rank barrier: every rank holds the full `out`.
//
// Stores to peers are plain 16-byte global stores; TMA reads only local operands
// and never multicasts.  Waits are bounded: on timeout the kernel records a status word,
// still meets every grid barrier and returns.
#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"
#include "launchers.h"
#include "tma_host.h"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace s0 {
namespace tpf {

using bf16 = __nv_bfloat16;
constexpr int BM = 128, BK = 64;
// warp roles: 0-3 epilogue (TMEM lane quadrants), 4 MMA issue, 5 TMA loads
constexpr int NT = 192, EPI_WARPS = 4, MMA_WARP = 4, PROD_WARP = 5;
constexpr int EPI_C = 64;                                       // columns staged per epilogue pass
constexpr int EPI_LD = EPI_C + 8;                               // bf16 row stride of a staged row
constexpr int EPI_BYTES = BM * EPI_LD * 2;                      // 18 KB: each epilogue warp stages 32 rows

// phase 3 streams row blocks of the local receive slots through shared memory
constexpr int P3_STAGE = 64 * 1024, P3_NS = 3;

// Tile width BN (128 or 256 output columns): a 128 x 256 tile halves the operand bytes
// staged per FLOP, which the 128 x 128 tile spends faster than shared memory refills.
template <int BN>
struct Cfg {
  static constexpr int STAGE_BYTES = (BM + BN) * BK * 2;       // 32 or 48 KB
  static constexpr int NS = BN == 256 ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;                     // two accumulators
  static constexpr size_t SMEM = 1024 + (size_t)NS * STAGE_BYTES + EPI_BYTES;
};

__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(mbar)), "r"(bytes)
               : "memory");
}
// 2-D tiled TMA load (no multicast) of the box at (x = k, y = row) into swizzled shared memory
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_u32(mbar))
      : "memory");
}

// untiled bulk copy (no multicast) of `bytes` contiguous local global bytes into shared memory
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(tc::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(tc::smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block 0's first `world` threads signal peer t and wait for peer t's signal of `phase`.
__device__ void xbar(const TpfArgs& a, int phase) {
  const int t = threadIdx.x;
  __threadfence_system();
  __syncthreads();
  if (t < a.world && t != a.rank) {
    st_release_sys(a.flags[t] + phase * TPF_MAXW + a.rank, a.seq);
    const int* mine = a.flags[a.rank] + phase * TPF_MAXW + t;
    long long it = 0;
    while (ld_acquire_sys(mine) < a.seq) {
      if (++it > a.spin_limit) {
        atomicExch(a.abort, 1);
        atomicExch(a.status, 100 + phase);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

template <int BN>
__global__ void __launch_bounds__(NT, 1)
    tp_gemm_allreduce_k(TpfArgs a, const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB) {
  using C = Cfg<BN>;
  constexpr int NS = C::NS, STAGE_BYTES = C::STAGE_BYTES;
  cg::grid_group grid = cg::this_grid();
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2], p3bar[P3_NS];
  __shared__ uint32_t tslot;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  bf16* stile = reinterpret_cast<bf16*>(base + (size_t)NS * STAGE_BYTES);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (a.stamps && blockIdx.x == 0 && tid == 0) a.stamps[0] = globaltimer();
  if (warp == 0) tc::tmem_alloc(&tslot, C::TMEM_COLS);
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < P3_NS; ++i) tc::mbar_init(&p3bar[i], 1);
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
  const uint32_t idesc = tc::idesc_bf16(BM, BN);
  const int tiles_m = a.M / BM, tiles_n = a.N / BN, nk = a.K / BK;
  const int ntiles = tiles_m * tiles_n;
  bool ok = true;
  // ---- phase 1: tiles -> the owners' receive slots (warp-specialised pipeline) --------------
  if (warp == PROD_WARP) {
    // one thread streams every chunk of this CTA's tiles with TMA: chunk g -> stage g % NS
    if (lane == 0) {
      long g = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int tm = t / tiles_n, tn = t % tiles_n;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % NS);
          const long u = g / NS;
          if (u > 0) ok = tc::mbar_wait(&empty[s], (uint32_t)((u - 1) & 1)) && ok;
          unsigned char* sA = base + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sA, &tmA, kt * BK, tm * BM, &full[s]);
          tma_load_2d(sA + BM * 128, &tmB, kt * BK, tn * BN, &full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      long g = 0;
      int j = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2) ok = tc::mbar_wait(&acc_empty[b], (uint32_t)(((j >> 1) - 1) & 1)) && ok;
        tc::fence_after_sync();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % NS);
          ok = tc::mbar_wait(&full[s], (uint32_t)((g / NS) & 1)) && ok;
          tc::fence_after_sync();
          unsigned char* sA = base + s * STAGE_BYTES;
          unsigned char* sB = sA + BM * 128;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            tc::mma_bf16(acc, tc::desc_sw128(sA, ks), tc::desc_sw128(sB, ks), idesc, (kt | ks) != 0);
          tc::commit(&empty[s]);
        }
        tc::commit(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps: TMEM buffer -> bf16 -> this warp's 32 staged rows (EPI_C columns per
    // pass) -> 16-byte stores of whole 128-byte row segments
    bf16* my = stile + (size_t)warp * 32 * EPI_LD;
    int j = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
      const int tm = t / tiles_n, tn = t % tiles_n, b = j & 1;
      ok = tc::mbar_wait(&acc_full[b], (uint32_t)((j >> 1) & 1)) && ok;
      tc::fence_after_sync();
      const int owner = tm % a.world, lt = tm / a.world;
      __nv_bfloat16* dst = a.recv[owner] + ((size_t)a.rank * a.rows_own + (size_t)lt * BM + 32 * warp) * a.N +
                           (size_t)tn * BN;
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += EPI_C) {
#pragma unroll
        for (int c0 = 0; c0 < EPI_C; c0 += 16) {
          float v[16];
          tc::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(b * BN + cc + c0), v);
          uint4* d = reinterpret_cast<uint4*>(my + lane * EPI_LD + c0);
          d[0] = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                            pack_bf16(v[6], v[7]));
          d[1] = make_uint4(pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]), pack_bf16(v[12], v[13]),
                            pack_bf16(v[14], v[15]));
        }
        if (cc + EPI_C == BN) {
          tc::fence_before_sync();
          tc::mbar_arrive(&acc_empty[b]);         // this thread's reads of buffer b are done
        }
        __syncwarp();
#pragma unroll
        for (int i = lane; i < 32 * (EPI_C / 8); i += 32) {
          const int r = i / (EPI_C / 8), c8 = i % (EPI_C / 8);
          *reinterpret_cast<uint4*>(dst + (size_t)r * a.N + cc + c8 * 8) =
              *reinterpret_cast<const uint4*>(my + r * EPI_LD + c8 * 8);
        }
        __syncwarp();
      }
    }
  }
  if (!ok) atomicExch(a.status, 1);
  if (a.stamps) {
    __syncthreads();
    if (tid == 0) a.stamps[4 + blockIdx.x] = globaltimer();
  }
  __threadfence_system();
  grid.sync();
  if (a.stamps && blockIdx.x == 0 && tid == 0) a.stamps[1] = globaltimer();
  // ---- phase 2: every rank's additions have landed ----------------------------------------
  if (blockIdx.x == 0) xbar(a, 0);
  grid.sync();
  if (!*((volatile int*)a.abort)) {
    // ---- phase 3: sum the partials of the owned rows, all-gather them as bf16 -------------
    // The owned rows are cut into blocks of `rb` rows (rb divides 128, so a block is one
    // contiguous range of every slot and of the output).  Thread 0 bulk-copies the world
    // slots' rows of a block into one of P3_NS shared-memory stages (the phase-1 operand
    // stages, idle now); all threads sum the slots in fp32, round to bf16 and store the block
    // into every rank's output.  The copies read only this GPU's receive buffer.
    const int row_bytes = a.N * 2;
    int rb = 128;
    while (rb > 1 && rb * row_bytes * a.world > P3_STAGE) rb >>= 1;
    const int owned_rows = (int)((tiles_m - a.rank + a.world - 1) / a.world) * BM;
    const int nblk = owned_rows / rb;
    const int blk_bytes = rb * row_bytes;                 // one slot's share of a block
    const int blk_c = blk_bytes / 16;                     // 16-byte chunks per slot share
    const __nv_bfloat16* rv = a.recv[a.rank];
    auto issue = [&](int i, int st) {                     // block i of this CTA -> stage st
      const int blk = blockIdx.x + i * gridDim.x;
      unsigned char* sm = base + (size_t)st * P3_STAGE;
      mbar_expect_tx(&p3bar[st], (uint32_t)(blk_bytes * a.world));
      for (int k = 0; k < a.world; ++k)
        bulk_load(sm + (size_t)k * blk_bytes, rv + ((size_t)k * a.rows_own + (size_t)blk * rb) * a.N,
                  (uint32_t)blk_bytes, &p3bar[st]);
    };
    const int my_blocks = nblk > (int)blockIdx.x ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (tid == 0) {
      // the slots were written by generic-proxy stores (ours and the peers', ordered by the
      // barrier's acquire); order them before the async-proxy reads
      asm volatile("fence.proxy.async.global;" ::: "memory");
      for (int i = 0; i < P3_NS && i < my_blocks; ++i) issue(i, i);
    }
    bool ok3 = true;
    for (int i = 0; i < my_blocks; ++i) {
      const int st = i % P3_NS;
      ok3 = tc::mbar_wait(&p3bar[st], (uint32_t)((i / P3_NS) & 1)) && ok3;
      const unsigned char* sm = base + (size_t)st * P3_STAGE;
      const int lrow0 = (blockIdx.x + i * gridDim.x) * rb;
      const size_t row0 = (size_t)(a.rank + (lrow0 / BM) * a.world) * BM + lrow0 % BM;
      for (int c = tid; c < blk_c; c += NT) {
        float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < a.world; ++k) {
          const uint4 q = *reinterpret_cast<const uint4*>(sm + (size_t)k * blk_bytes + (size_t)c * 16);
          const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_bf16(w4[e]);
            acc8[2 * e] += f.x;
            acc8[2 * e + 1] += f.y;
          }
        }
        const uint4 o = make_uint4(pack_bf16(acc8[0], acc8[1]), pack_bf16(acc8[2], acc8[3]),
                                   pack_bf16(acc8[4], acc8[5]), pack_bf16(acc8[6], acc8[7]));
        for (int k = 0; k < a.world; ++k) {
          const int kk = (a.rank + k) % a.world;   // stagger the targets across ranks
          reinterpret_cast<uint4*>(a.out[kk] + row0 * a.N)[c] = o;
        }
      }
      __syncthreads();                               // stage st fully read
      if (tid == 0 && i + P3_NS < my_blocks) issue(i + P3_NS, st);
    }
    if (!ok3) atomicExch(a.status, 2);
  }
  __threadfence_system();
  grid.sync();
  if (a.stamps && blockIdx.x == 0 && tid == 0) a.stamps[2] = globaltimer();
  // ---- phase 4: every output row delivered everywhere -------------------------------------
  if (blockIdx.x == 0) xbar(a, 1);
  if (a.stamps && blockIdx.x == 0 && tid == 0) a.stamps[3] = globaltimer();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace tpf
}  // namespace s0

namespace {
template <int BN>
int launch_bn(const TpfArgs& a, int sms, cudaStream_t st) {
  using namespace s0::tpf;
  using C = Cfg<BN>;
  auto* kern = tp_gemm_allreduce_k<BN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, C::SMEM);
  if (per_sm < 1) return -2;
  // one CTA per SM: its shared memory holds the pipeline and its accumulators fill the TMEM
  const long tiles = (long)(a.M / BM) * (a.N / BN);
  const int grid = (int)(tiles < sms ? tiles : sms);
  // operand tensor maps: [rows, K] bf16, boxes of 64 K-elements (128-byte rows) x `box_rows`,
  // 128-byte swizzle -- the K-major SW128 layout the MMA descriptors expect
  CUtensorMap tmA, tmB;
  auto encode = [](CUtensorMap* m, const void* ptr, int rows, int K, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const auto enc = s0::tensor_map_encoder();
    if (!enc) return CUDA_ERROR_NOT_FOUND;
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.Bt)) % 16) return -3;
  if (encode(&tmA, a.A, a.M, a.K, BM) != CUDA_SUCCESS || encode(&tmB, a.Bt, a.N, a.K, BN) != CUDA_SUCCESS) return -4;
  TpfArgs args = a;
  void* kargs[] = {&args, &tmA, &tmB};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, dim3(grid), dim3(NT), kargs, C::SMEM, st);
  return e == cudaSuccess ? 0 : (int)e;
}
}  // namespace

int tp_gemm_allreduce_launch(const TpfArgs& a, int sms, cudaStream_t st) {
  using namespace s0::tpf;
  if (a.M % BM || a.N % 128 || a.K % BK || a.K <= 0 || a.world < 1 || a.world > TPF_MAXW) return -1;
  if ((long)a.N * 2 * a.world > P3_STAGE) return -5;   // one row of every slot must fit a phase-3 stage
  return a.N % 256 == 0 ? launch_bn<256>(a, sms, st) : launch_bn<128>(a, sms, st);
}
