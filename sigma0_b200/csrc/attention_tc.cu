// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Same contract as attn_fwd_k in attention.cu (causal, sliding window, decode offsets,
// per-key position tables, per-entry query offsets; o and the base-2 row log-sum-exp
// for the shared backward), for the layouts [B, L, nh, HD] with HD in {64, 128}.
//
// One CTA per (128 query rows, head, batch), 8 warps with fixed roles:
//   warp 0     TMA producer: the Q tile once, then K and V blocks of 128 keys into a
//              two-stage ring (4-D tensor maps over the strided [B, L, nh, HD] tensors,
//              boxes of 64 head-dim elements x 128 rows, 128-byte swizzle, no multicast;
//              rows past the end read as zeros);
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM accumulators
//              (128 x 128 fp32), then O += P_{j-1} V_{j-1} into the TMEM output (128 x HD)
//              -- P is the K-major A operand in shared memory, V the MN-major B operand
//              straight from its TMA tile (rows of keys, 64 head-dim elements per 128-byte
//              row: stride between 8-key groups 1024 B, between 64-column boxes 16 KB);
//   warp 2     allocates / frees the tensor memory;
//   warps 4-7  softmax: thread t owns query row t (= TMEM lane t): reads its S row with
//              tcgen05.ld, masks, takes the row max and exp2, writes its P row (bf16,
//              swizzled) to shared memory, and rescales its O row in TMEM only when the
//              running max grew by more than 8 (log2 units; the stale max keeps every p
//              <= 256, exact in the final normalisation) -- then the epilogue: O / l to
//              bf16 global rows and the log-sum-exp.
// The S double buffer lets QK_{j+1} run on the tensor cores while the softmax of block j
// runs on the CUDA cores.  Every mbarrier wait is bounded; a timeout sets *status.  No
// asynchronous arrive is left outstanding at exit (the grid runs in several waves, and a
// late arrive would land on the barriers of the next CTA on the SM): a stage-release commit
// is issued only when a later load waits for it, and the MMA thread waits for its last
// commit before leaving.
#include <cuda.h>
#include <cuda_bf16.h>
#include <math_constants.h>

#include "common.cuh"
#include "launchers.h"
#include "tma_host.h"
#include "tc_common.cuh"

namespace s0 {
namespace attn_tc {

using bf16 = __nv_bfloat16;
constexpr int BQ = 128, BKV = 128, NT = 256;
constexpr int BOX = 128 * 128;                 // bytes of one 64-column x 128-row SW128 box

template <int HD>
struct Cfg {
  static constexpr int NB = HD / 64;           // boxes per 128-row tile
  static constexpr int TILE = NB * BOX;        // Q, K or V tile bytes
  static constexpr int SMEM = 1024 + TILE * 5 + 2 * BOX;   // Q, 2 x K, 2 x V, P (128 x 128 bf16)
  static constexpr int TMEM_COLS = 512;        // 2 x S (128 columns) + O (HD columns)
};

__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(mbar)), "r"(bytes)
               : "memory");
}
// 4-D tiled TMA load (no multicast): box (64, 1, 128, 1) at (d0, head, row, batch)
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int d0, int h, int row, int b,
                                            uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(d0), "r"(h), "r"(row), "r"(b), "r"(tc::smem_u32(mbar))
      : "memory");
}
// MN-major SWIZZLE_128B descriptor: rows of 64 N-elements (128 B), 8-row K groups 1024 B apart,
// consecutive 64-element N chunks `lbo` bytes apart
__device__ __forceinline__ uint64_t desc_mn_sw128(const void* tile, uint32_t lbo) {
  const uint32_t addr = tc::smem_u32(tile);
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool visible(int key, int kp, int qpos, int Lk, int window) {
  return key < Lk && kp <= qpos && (window <= 0 || kp > qpos - window);
}

template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_fwd_tc_k(AttnArgs a, const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv) {
  using K = Cfg<HD>;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full, o_done;
  __shared__ uint32_t tslot;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  unsigned char* sQ = base;
  unsigned char* sK = sQ + K::TILE;             // [2][TILE]
  unsigned char* sV = sK + 2 * K::TILE;         // [2][TILE]
  unsigned char* sP = sV + 2 * K::TILE;         // [2 boxes] = 128 rows x 128 keys bf16
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qoff = a.qoff ? a.qoff[b] : a.q_offset;
  const int* kp = a.kpos ? a.kpos + (long)b * a.Lk : nullptr;
  const int qlo = qoff + q0;
  int kb0 = 0, kb1 = (a.Lk + BKV - 1) / BKV;
  if (!kp) {
    const int hi = min(a.Lk, qlo + BQ);
    const int lo = a.window > 0 ? max(0, qlo - a.window + 1) : 0;
    kb0 = lo / BKV;
    kb1 = hi > lo ? (hi + BKV - 1) / BKV : kb0;
  }
  const int n = kb1 - kb0;

  if (warp == 2) tc::tmem_alloc(&tslot, K::TMEM_COLS);
  if (tid == 0) {
    tc::mbar_init(&q_full, 1);
    tc::mbar_init(&p_full, 128);
    tc::mbar_init(&o_done, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&kv_full[i], 1);
      tc::mbar_init(&kv_empty[i], 1);
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&s_empty[i], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tslot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      mbar_expect_tx(&q_full, K::TILE);
      for (int x = 0; x < K::NB; ++x) tma_load_4d(sQ + x * BOX, &tq, 64 * x, h, q0, b, &q_full);
      for (int i = 0; i < n; ++i) {
        const int st = i & 1, key0 = (kb0 + i) * BKV;
        if (i >= 2) ok = tc::mbar_wait(&kv_empty[st], (uint32_t)(((i - 2) >> 1) & 1)) && ok;
        mbar_expect_tx(&kv_full[st], 2 * K::TILE);
        for (int x = 0; x < K::NB; ++x) {
          tma_load_4d(sK + st * K::TILE + x * BOX, &tk, 64 * x, h, key0, b, &kv_full[st]);
          tma_load_4d(sV + st * K::TILE + x * BOX, &tv, 64 * x, h, key0, b, &kv_full[st]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      const uint32_t id_qk = tc::idesc_bf16(BQ, BKV);
      const uint32_t id_pv = tc::idesc_bf16(BQ, HD) | (1u << 16);      // B (V) MN-major
      const uint32_t tO = tmem + 256;
      auto pv = [&](int j) {                                           // O += P_j V_j
        ok = tc::mbar_wait(&p_full, (uint32_t)(j & 1)) && ok;
        tc::fence_after_sync();
        const unsigned char* v = sV + (j & 1) * K::TILE;
#pragma unroll
        for (int ks = 0; ks < BKV / 16; ++ks)
          tc::mma_bf16(tO, tc::desc_sw128(sP + (ks >> 2) * BOX, ks & 3), desc_mn_sw128(v + ks * 2048, BOX), id_pv,
                       j > 0 || ks > 0);
        tc::commit(&o_done);
        // only the loads of block j + 2 wait for this stage: a commit nobody waits for could
        // still be in flight when the CTA exits and land on the next CTA's barriers
        if (j + 2 < n) tc::commit(&kv_empty[j & 1]);
      };
      ok = tc::mbar_wait(&q_full, 0) && ok;
      for (int i = 0; i < n; ++i) {
        const int st = i & 1;
        ok = tc::mbar_wait(&kv_full[st], (uint32_t)((i >> 1) & 1)) && ok;
        if (i >= 2) ok = tc::mbar_wait(&s_empty[st], (uint32_t)(((i - 2) >> 1) & 1)) && ok;
        tc::fence_after_sync();
        const unsigned char* kt = sK + st * K::TILE;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          tc::mma_bf16(tmem + st * 128, tc::desc_sw128(sQ + (ks >> 2) * BOX, ks & 3),
                       tc::desc_sw128(kt + (ks >> 2) * BOX, ks & 3), id_qk, ks > 0);
        tc::commit(&s_full[st]);
        if (i >= 1) pv(i - 1);
      }
      pv(n - 1);
      ok = tc::mbar_wait(&o_done, (uint32_t)((n - 1) & 1)) && ok;     // every MMA retired before exit
    }
    __syncwarp();
  } else if (warp >= 4) {
    // softmax / epilogue: row r = TMEM lane r
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
    const int row = q0 + r, qpos = qoff + row;
    float m_run = -CUDART_INF_F, l = 0.f;
    for (int i = 0; i < n; ++i) {
      const int st = i & 1, key0 = (kb0 + i) * BKV;
      ok = tc::mbar_wait(&s_full[st], (uint32_t)((i >> 1) & 1)) && ok;
      tc::fence_after_sync();
      float s[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 16; ++c) tc::tmem_ld16(tmem + lanes + st * 128 + c * 16, s + c * 16);
      tc::fence_before_sync();
      tc::mbar_arrive(&s_empty[st]);
      const bool full = !kp && key0 + BKV - 1 <= qlo && key0 + BKV <= a.Lk &&
                        (a.window <= 0 || key0 > qlo + BQ - 1 - a.window);
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int j = 0; j < BKV; ++j) {
        float x = s[j] * a.scale_log2;
        if (!full) {
          const int key = key0 + j;
          const int kpj = kp ? (key < a.Lk ? __ldg(kp + key) : 0x7fffffff) : key;
          if (!visible(key, kpj, qpos, a.Lk, a.window)) x = -CUDART_INF_F;
        }
        s[j] = x;
        mx = fmaxf(mx, x);
      }
      bool rescale = false;
      float alpha = 1.f;
      if (m_run == -CUDART_INF_F) {
        m_run = mx;                                    // nothing of weight accumulated yet
      } else if (mx > m_run + 8.f) {
        alpha = exp2f(m_run - mx);
        l *= alpha;
        m_run = mx;
        rescale = true;
      }
      const float bias = m_run == -CUDART_INF_F ? 0.f : m_run;
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < BKV; ++j) {
        const float p = exp2f(s[j] - bias);
        s[j] = p;
        ps += p;
      }
      l += ps;
      if (i > 0) {
        ok = tc::mbar_wait(&o_done, (uint32_t)((i - 1) & 1)) && ok;   // PV_{i-1} done: P free, O stable
        tc::fence_after_sync();
      }
      if (rescale) {
#pragma unroll
        for (int c = 0; c < HD / 16; ++c) {
          float o[16];
          tc::tmem_ld16(tmem + lanes + 256 + c * 16, o);
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] *= alpha;
          tmem_st16(tmem + lanes + 256 + c * 16, o);
        }
        tmem_wait_st();
      }
      // P row -> shared memory (K-major SW128: keys 0-63 in box 0, 64-127 in box 1)
#pragma unroll
      for (int c = 0; c < BKV / 8; ++c) {
        const uint4 v = make_uint4(pack_bf16(s[8 * c], s[8 * c + 1]), pack_bf16(s[8 * c + 2], s[8 * c + 3]),
                                   pack_bf16(s[8 * c + 4], s[8 * c + 5]), pack_bf16(s[8 * c + 6], s[8 * c + 7]));
        *reinterpret_cast<uint4*>(sP + (c >> 3) * BOX + r * 128 + ((((c & 7) ^ (r & 7)) & 7) << 4)) = v;
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::mbar_arrive(&p_full);
    }
    // epilogue
    bf16* og = a.o + b * a.so_b + (long)row * a.so_l + h * a.so_h;
    if (n > 0) {
      ok = tc::mbar_wait(&o_done, (uint32_t)((n - 1) & 1)) && ok;
      tc::fence_after_sync();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int c = 0; c < HD / 16; ++c) {
      float o[16];
      if (n > 0) {
        tc::tmem_ld16(tmem + lanes + 256 + c * 16, o);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e] = 0.f;
      }
      if (row < a.Lq) {
        uint4* d = reinterpret_cast<uint4*>(og + c * 16);
        d[0] = make_uint4(pack_bf16(o[0] * inv, o[1] * inv), pack_bf16(o[2] * inv, o[3] * inv),
                          pack_bf16(o[4] * inv, o[5] * inv), pack_bf16(o[6] * inv, o[7] * inv));
        d[1] = make_uint4(pack_bf16(o[8] * inv, o[9] * inv), pack_bf16(o[10] * inv, o[11] * inv),
                          pack_bf16(o[12] * inv, o[13] * inv), pack_bf16(o[14] * inv, o[15] * inv));
      }
    }
    if (row < a.Lq) a.lse[((long)b * a.nh + h) * a.Lq + row] = l > 0.f ? m_run + log2f(l) : CUDART_INF_F;
  }
  if (!ok && a.status) atomicExch(a.status, 1);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, K::TMEM_COLS);
}

// [B, L, nh, HD] bf16 with element strides (sb, sl, sh, 1) -> 4-D map, box (64, 1, 128, 1)
static int encode(CUtensorMap* m, const void* ptr, int B, int L, int nh, int HD, long sb, long sl, long sh) {
  const cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)nh, (cuuint64_t)L, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sl * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, 1, 128, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const auto enc = s0::tensor_map_encoder();
  if (!enc) return -4;
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : -4;
}

template <int HD>
int launch(const AttnArgs& a, cudaStream_t st) {
  using K = Cfg<HD>;
  CUtensorMap tq, tk, tv;
  if (encode(&tq, a.q, a.B, a.Lq, a.nh, HD, a.sq_b, a.sq_l, a.sq_h) ||
      encode(&tk, a.k, a.B, a.Lk, a.nh, HD, a.sk_b, a.sk_l, a.sk_h) ||
      encode(&tv, a.v, a.B, a.Lk, a.nh, HD, a.sv_b, a.sv_l, a.sv_h))
    return -4;
  // one CTA per SM: it holds 512 tensor-memory columns
  const int smem = K::SMEM > 120 * 1024 ? K::SMEM : 120 * 1024;
  cudaFuncSetAttribute(attn_fwd_tc_k<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((a.Lq + BQ - 1) / BQ, a.nh, a.B);
  attn_fwd_tc_k<HD><<<grid, NT, smem, st>>>(a, tq, tk, tv);
  return (int)cudaGetLastError();
}

}  // namespace attn_tc
}  // namespace s0

int attn_fwd_tc_launch(const AttnArgs& a, int hd, cudaStream_t st) {
  if (a.Lq <= 0 || a.Lk <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) % 16)
    return -3;
  if (hd == 64) return s0::attn_tc::launch<64>(a, st);
  if (hd == 128) return s0::attn_tc::launch<128>(a, st);
  return -1;
}
