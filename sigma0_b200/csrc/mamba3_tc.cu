// Mamba-3 SISO chunked SSD on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Forward and backward as ONE kernel each per layer: a CTA walks the chunks of one
// (sequence, head) in order -- forward from the first chunk, backward from the last -- and
// carries the recurrent state S (forward) or its gradient dS (backward), d_state x headdim in
// fp32, in tensor memory from chunk to chunk.  The per-chunk state contributions, the
// state-passing scan and the chunk scan of a chunk-parallel formulation become one pass with
// no state round trip through HBM.  Replaces the reference's chunk_state / state-passing /
// chunk_scan kernels and their backward (src/base_model/models/mamba3_pallas.py:199-419,
// src/base_model/kernels/mamba3_cuda/src/siso_state_scan.cu:133-255).
//
// Forward, per chunk of CS = 64 tokens (8 warps, lockstep phases; thread 0 issues TMA/MMAs):
//   loads   Bn | Cn tiles (TMA, 128-byte swizzle) once the previous chunk's MMAs have read the
//           tiles; V (TMA), the angle rates and dt / decay / gate rows (cp.async) one chunk
//           ahead into a two-stage ring
//   B       row scalars (decay cumsum, trapezoid weights), rotary angles carried across chunks
//   C       Q = rope(Cn + C_bias), K = rope(Bn + B_bias) * scale built in place over the tiles;
//           w*V for the state update
//   D       S_in: TMEM -> bf16 swizzled image (bulk-copied to HBM for the backward), then the
//           TMEM state is scaled by the chunk decay
//   F       MMAs: Sc = Q K^T (M=64), Yoff = Q S_in^T (M=64), state += K^T (w V) (M=128)
//   G       P = mask(Sc * exp(cum_l - cum_s)) -> bf16 tile
//   H       MMA: Ypv = P V
//   I       y = (Ypv + exp(cum_l) Yoff + (D + gamma qk) V) * silu(z) -> swizzled tile -> TMA store
// Accumulators: M=64 tiles keep row r in TMEM lane 32*(r/16) + r%16 and are read with the
// 16x256b shape (mma.sync C-fragment layout); the state is an M=128 tile (lane = state row n).
// No TMA load uses cluster multicast: every tile comes from this GPU's own memory.
// Every mbarrier wait is bounded: on a timeout the CTA records the failure in a status word,
// waits (bounded) for its copies in flight, frees its tensor memory and returns.
#include <cuda.h>

#include "common.cuh"
#include "launchers.h"
#include "tc_common.cuh"
#include "tma_host.h"

namespace s0 {
namespace m3tc {

using bf16 = __nv_bfloat16;
constexpr int CS = 64, N = 128, P = 64, R = 32;
constexpr int NT = 256;
constexpr float TWO_PI_F = 6.28318530717958647692f;
constexpr int BOX = 64 * 128;               // one SW128 box: 64 rows x 64 bf16
constexpr uint32_t TM_S = 0, TM_YOFF = 64, TM_PV = 128, TM_ST = 192, TM_COLS = 256;
constexpr long long WAIT_LIMIT = 1LL << 22;  // polls of try_wait (each may block ~us): seconds

// stage of the two-stage ring (one per chunk in flight): V tile, rates, dt / adt / sig rows
struct __align__(1024) Stage {
  unsigned char v[BOX];          // V [s][p] SW128
  float rate[CS * R];            // [s][r]
  float dt[CS + 4], sig[CS + 4], adt[CS];
};
struct __align__(1024) Smem {
  unsigned char bn[2 * BOX];     // Bn -> K (two 64-column boxes)
  unsigned char cn[2 * BOX];     // Cn -> Q
  unsigned char sin_[2 * BOX];   // S_in image: rows n (128) x 64 p, SW128
  unsigned char p[BOX];          // P [l][s]; later the y tile for the TMA store
  unsigned char wv[BOX];         // w * V [s][p]
  Stage stage[2];
  float cum[CS], gam[CS], scl[CS], qkp[2][CS];
  float seg[8 * 32], th[R], thnext[R];
  float cb[N], bb[N];
  uint64_t bc_full, vs_full[2], mma1, mma2;
  uint32_t tslot;
};
static_assert(sizeof(Smem) + 1024 <= 116736, "forward shared memory must allow two CTAs per SM");

struct FwdArgs {
  const bf16* proj;
  const float *dt, *adt, *sig, *rate;      // dt / adt / sig: [B, nh, L] with row stride lds
  const float *Bb, *Cb, *D;
  bf16* states;                            // [B, nh, nc] images of S_in (16 KB each) or null
  float* theta0;                           // [B, nh, nc, R] angle at each chunk start, or null
  const float* s0;                         // [B, nh, nseg, P, N] initial state of each segment or null
  const float* th_in;                      // [B, nh, nseg, R] initial angle of each segment or null
  float* fin;                              // [B, nh, nseg, P, N] final state of each segment or null
  float* thf;                              // [B, nh, nseg, R] final angle of each segment or null
  int* status;
  int B, L, nh, ldp, lds, nc;
  int cps, nseg, seg_lo, seg_hi;           // chunks per segment; this launch walks segments [lo, hi)
};

__device__ __forceinline__ uint32_t swz(int row, int chunk16) {   // byte offset in an SW128 tile
  return (uint32_t)(row * 128 + (((chunk16 ^ row) & 7) << 4));
}
__device__ __forceinline__ uint32_t frag_off(int row, int col) {   // bf16 (row, col) in an SW128 tile
  return (uint32_t)(col >> 6) * BOX + swz(row, (col >> 3) & 7) + (uint32_t)(col & 7) * 2;
}

// theta table [64][32] fp32 with an xor swizzle on groups of 4 angles, so that the epilogue's
// reads (8 rows x 4 angles per warp) and the build's float4 reads hit distinct banks
__device__ __forceinline__ int th_idx(int row, int r) { return row * R + (r ^ ((row & 7) << 2)); }

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t ph) { return tc::mbar_wait(bar, ph, WAIT_LIMIT); }

// loads of chunk c (the i-th of this walk) into stage i & 1 (V, rates, scalars); warp 0 calls it
__device__ __forceinline__ void load_stage(Smem& sm, const FwdArgs& a, const CUtensorMap* tm_proj, int b, int h,
                                           int c, int i, int lane) {
  Stage& st = sm.stage[i & 1];
  uint64_t* bar = &sm.vs_full[i & 1];
  const int t0 = c * CS;
  if (lane == 0) {
    tc::mbar_expect_tx(bar, BOX);
    tc::tma_load_3d(st.v, tm_proj, a.nh * P + h * P, t0, b, bar);
  }
  const float* rate = a.rate + (size_t)b * a.L * R;
  for (int i = lane; i < CS * R / 4; i += 32) {
    const int r = i >> 3, q = i & 7, t = t0 + r;
    const bool ok = t < a.L;
    cp_async16(st.rate + r * R + q * 4, rate + (size_t)(ok ? t : 0) * R + q * 4, ok ? 16 : 0);
  }
  const size_t row = ((size_t)b * a.nh + h) * a.lds;
  for (int i = lane; i < 3 * (CS + 1); i += 32) {
    const int which = i / (CS + 1), k = i % (CS + 1), t = t0 + k;
    if (which == 2 && k == CS) continue;
    const bool ok = t < a.L;
    const float* src = which == 0 ? a.dt : which == 1 ? a.sig : a.adt;
    float* dst = which == 0 ? st.dt : which == 1 ? st.sig : st.adt;
    cp_async4(dst + k, src + row + (ok ? t : 0), ok ? 4 : 0);
  }
  tc::cp_async_mbar_arrive(bar);
}

__global__ void __launch_bounds__(NT, 2)
    m3_fwd_tc_k(FwdArgs a, const __grid_constant__ CUtensorMap tm_bc, const __grid_constant__ CUtensorMap tm_proj,
                const __grid_constant__ CUtensorMap tm_y) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nsl = a.seg_hi - a.seg_lo;
  const int bh = blockIdx.x / nsl, seg = a.seg_lo + blockIdx.x % nsl, b = bh / a.nh, h = bh % a.nh;
  const size_t slot = (size_t)bh * a.nseg + seg;          // this (sequence, head, segment)
  const int nc = a.nc, cb = seg * a.cps, ce = min(nc, cb + a.cps);

  if (warp == 0) tc::tmem_alloc(&sm.tslot, TM_COLS);
  if (tid == 0) {
    tc::mbar_init(&sm.bc_full, 1);
    tc::mbar_init(&sm.vs_full[0], 33);
    tc::mbar_init(&sm.vs_full[1], 33);
    tc::mbar_init(&sm.mma1, 1);
    tc::mbar_init(&sm.mma2, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < N; i += NT) {
    sm.cb[i] = a.Cb[h * N + i];
    sm.bb[i] = a.Bb[h * N + i];
  }
  if (tid < R) sm.th[tid] = a.th_in ? a.th_in[slot * R + tid] : 0.f;
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tslot;
  const int q = warp & 3, half = warp >> 2;              // TMEM lane quadrant, column half
  const uint32_t lane_base = (uint32_t)(32 * q) << 16;
  const int g = lane >> 2, tq = lane & 3;
  const int r0 = 16 * q + g, r1 = r0 + 8;                // rows of this thread's M=64 fragments
  // Q / K build: thread (half, bu) owns 8-column chunk bch of box `half` for rows bu/8 + 16k
  const int bu = (warp & 3) * 32 + lane, bch = bu & 7;
  float cbr[8], bbr[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    cbr[j] = sm.cb[64 * half + 8 * bch + j];
    bbr[j] = sm.bb[64 * half + 8 * bch + j];
  }

  // initial state: S^T rows n (lanes) x p (columns) in TMEM
  if (a.s0) {
    float v[32];
    const int n = 32 * q + lane;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = a.s0[(slot * P + 32 * half + j) * N + n];
    tc::tmem_st32(tmem + lane_base + TM_ST + 32 * half, v);
    tc::tmem_wait_st();
  }
  if (warp == 0) {
    if (lane == 0) {
      tc::mbar_expect_tx(&sm.bc_full, 4 * BOX);
      for (int k = 0; k < 4; ++k)
        tc::tma_load_3d((k < 2 ? sm.bn : sm.cn) + (k & 1) * BOX, &tm_bc, 64 * k, cb * CS, b, &sm.bc_full);
    }
    load_stage(sm, a, &tm_proj, b, h, cb, 0, lane);
  }
  const float Dh = a.D[h];
  bool ok = true;
  bool store_pending = false;                             // thread 0: bulk stores in flight
  int bc_loads = 1, vs_loads = 1;                         // loads issued so far (chunk count)

  for (int c = cb; c < ce; ++c) {
    const int t0 = c * CS, i = c - cb;                   // i: position in this walk
    Stage& st = sm.stage[i & 1];
    ok = wait(&sm.vs_full[i & 1], (i >> 1) & 1) && ok;
    if (warp == 0 && c + 1 < ce) load_stage(sm, a, &tm_proj, b, h, c + 1, i + 1, lane);
    if (c + 1 < ce) vs_loads = i + 2;
    // ---- B: row scalars and rotary angles ------------------------------------------------
    if (tid < CS) {
      const float d0 = st.dt[tid], s0_ = st.sig[tid], d1 = st.dt[tid + 1], s1 = st.sig[tid + 1];
      const float gm = d0 * s0_;
      sm.gam[tid] = gm;
      sm.scl[tid] = gm + d1 * (1.f - s1);
      float v = st.adt[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      sm.cum[tid] = v;
    }
    {   // theta prefix over rows: thread (r = lane, seg = warp) owns rows 8*seg .. 8*seg+7
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = warp * 8 + i;
        acc += st.rate[row * R + lane] * st.dt[row];
        st.rate[th_idx(row, lane)] = acc;                 // local prefix, in place (swizzled)
      }
      sm.seg[warp * 32 + lane] = acc;
    }
    __syncthreads();
    if (tid >= 32 && tid < CS) sm.cum[tid] += sm.cum[31];
    {
      float base = sm.th[lane];
      for (int s = 0; s < warp; ++s) base += sm.seg[s * 32 + lane];
#pragma unroll
      for (int i = 0; i < 8; ++i) st.rate[th_idx(warp * 8 + i, lane)] += base;   // theta (unreduced)
      if (warp == 7) {
        const float e = base + sm.seg[7 * 32 + lane];
        sm.thnext[lane] = e - TWO_PI_F * floorf(e * (1.f / TWO_PI_F));
      }
    }
    if (a.theta0 && tid < R) a.theta0[((size_t)bh * nc + c) * R + tid] = sm.th[tid];
    __syncthreads();
    const float cend = sm.cum[CS - 1];
    ok = wait(&sm.bc_full, i & 1) && ok;
    // ---- C: Q, K in place; qk diagonal; w * V --------------------------------------------
    // warps 0-3 take the rotated columns (box 0), warps 4-7 the rest, so no warp diverges on
    // the rotation; each thread keeps one 8-column chunk (its biases live in registers)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int row = (bu >> 3) + 16 * k;
      const uint32_t off = (uint32_t)half * BOX + swz(row, bch);
      uint4* qp = reinterpret_cast<uint4*>(sm.cn + off);
      uint4* kp = reinterpret_cast<uint4*>(sm.bn + off);
      const uint4 cv = *qp, bv = *kp;
      const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
      float cq[8], bk[8], qk = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 c2 = unpack_bf16(cw[j]), b2 = unpack_bf16(bw[j]);
        cq[2 * j] = c2.x + cbr[2 * j];
        cq[2 * j + 1] = c2.y + cbr[2 * j + 1];
        bk[2 * j] = b2.x + bbr[2 * j];
        bk[2 * j + 1] = b2.y + bbr[2 * j + 1];
        qk += cq[2 * j] * bk[2 * j] + cq[2 * j + 1] * bk[2 * j + 1];
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) qk += __shfl_xor_sync(0xffffffffu, qk, o);
      if (bch == 0) sm.qkp[half][row] = qk;
      if (half == 0) {
        const float4 th4 = *reinterpret_cast<const float4*>(st.rate + th_idx(row, 4 * bch));
        const float ths[4] = {th4.x, th4.y, th4.z, th4.w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float sn, cs;
          __sincosf(ths[m] - TWO_PI_F * floorf(ths[m] * (1.f / TWO_PI_F) + 0.5f), &sn, &cs);
          const float c0 = cq[2 * m], c1 = cq[2 * m + 1], b0 = bk[2 * m], b1 = bk[2 * m + 1];
          cq[2 * m] = c0 * cs - c1 * sn;
          cq[2 * m + 1] = c0 * sn + c1 * cs;
          bk[2 * m] = b0 * cs - b1 * sn;
          bk[2 * m + 1] = b0 * sn + b1 * cs;
        }
      }
      const float sc = sm.scl[row];
      *qp = make_uint4(pack_bf16(cq[0], cq[1]), pack_bf16(cq[2], cq[3]), pack_bf16(cq[4], cq[5]),
                       pack_bf16(cq[6], cq[7]));
      *kp = make_uint4(pack_bf16(bk[0] * sc, bk[1] * sc), pack_bf16(bk[2] * sc, bk[3] * sc),
                       pack_bf16(bk[4] * sc, bk[5] * sc), pack_bf16(bk[6] * sc, bk[7] * sc));
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * NT;
      const int row = i >> 3, ch = i & 7;
      const uint32_t off = swz(row, ch);
      const uint4 vv = *reinterpret_cast<const uint4*>(st.v + off);
      const float wr = __expf(cend - sm.cum[row]);
      const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16(vw[j]);
        o[j] = pack_bf16(f.x * wr, f.y * wr);
      }
      *reinterpret_cast<uint4*>(sm.wv + off) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    // ---- D: S_in -> bf16 image; TMEM state *= exp(chunk decay) ----------------------------
    if (tid == 0 && store_pending) tc::bulk_wait_read();   // last chunk's image copy has read sin_
    __syncthreads();
    {
      const int n = 32 * q + lane;
      float v[32];
      if (i > 0 || a.s0) {
        tc::fence_after_sync();
        tc::tmem_ld32(tmem + lane_base + TM_ST + 32 * half, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(sm.sin_ + swz(n, 4 * half + j)) =
            make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                       pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
      if (i > 0 || a.s0) {
        const float e = __expf(cend);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= e;
        tc::tmem_st32(tmem + lane_base + TM_ST + 32 * half, v);
        tc::tmem_wait_st();
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok);
    tc::fence_after_sync();
    if (!ok) break;
    // ---- F: MMAs on Q / K / S_in / wV ---------------------------------------------------------
    if (tid == 0) {
      if (a.states) {
        tc::bulk_store(a.states + ((size_t)bh * nc + c) * (N * P), sm.sin_, 2 * BOX);
        tc::bulk_commit();
        store_pending = true;
      }
      const uint32_t id64 = tc::idesc_bf16(64, 64);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16(tmem + TM_S, tc::desc_sw128(sm.cn + (ks >> 2) * BOX, ks & 3),
                     tc::desc_sw128(sm.bn + (ks >> 2) * BOX, ks & 3), id64, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16(tmem + TM_YOFF, tc::desc_sw128(sm.cn + (ks >> 2) * BOX, ks & 3),
                     tc::desc_mn_sw128(sm.sin_ + ks * 2048, BOX), id64 | tc::IDESC_B_MN, ks > 0);
      const uint32_t id128 = tc::idesc_bf16(128, 64) | tc::IDESC_A_MN | tc::IDESC_B_MN;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem + TM_ST, tc::desc_mn_sw128(sm.bn + ks * 2048, BOX),
                     tc::desc_mn_sw128(sm.wv + ks * 2048, BOX), id128, ks > 0 || i > 0 || a.s0 != nullptr);
      tc::commit(&sm.mma1);
    }
    // ---- G: P = masked decayed scores ---------------------------------------------------------
    ok = wait(&sm.mma1, i & 1) && ok;
    tc::fence_after_sync();
    if (tid == 0 && c + 1 < ce) {   // Q / K tiles consumed: fetch the next chunk's Bn | Cn
      tc::mbar_expect_tx(&sm.bc_full, 4 * BOX);
      for (int k = 0; k < 4; ++k)
        tc::tma_load_3d((k < 2 ? sm.bn : sm.cn) + (k & 1) * BOX, &tm_bc, 64 * k, t0 + CS, b, &sm.bc_full);
    }
    if (c + 1 < ce) bc_loads = i + 2;
    if (tid == 0 && store_pending) tc::bulk_wait_read();   // last chunk's y store has read p
    __syncthreads();
    {
      float v[16];
      tc::tmem_ld_frag32(tmem + lane_base + TM_S + 32 * half, v);
      const float cr0 = sm.cum[r0], cr1 = sm.cum[r1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s = 32 * half + 8 * j + 2 * tq;
        const float cs0 = sm.cum[s], cs1 = sm.cum[s + 1];
        const float p00 = s < r0 ? v[4 * j] * __expf(cr0 - cs0) : 0.f;
        const float p01 = s + 1 < r0 ? v[4 * j + 1] * __expf(cr0 - cs1) : 0.f;
        const float p10 = s < r1 ? v[4 * j + 2] * __expf(cr1 - cs0) : 0.f;
        const float p11 = s + 1 < r1 ? v[4 * j + 3] * __expf(cr1 - cs1) : 0.f;
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r0, s)) = pack_bf16(p00, p01);
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r1, s)) = pack_bf16(p10, p11);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // ---- H: Ypv = P V -------------------------------------------------------------------------
    if (tid == 0) {
      const uint32_t id = tc::idesc_bf16(64, 64) | tc::IDESC_B_MN;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem + TM_PV, tc::desc_sw128(sm.p, ks), tc::desc_mn_sw128(st.v + ks * 2048, BOX), id, ks > 0);
      tc::commit(&sm.mma2);
    }
    // z for the gate (global, bf16 pairs of this thread's fragment positions)
    uint32_t zr[8];
    {
      const bf16* zb = a.proj + ((size_t)b * a.L + t0) * a.ldp + h * P;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = 32 * half + 8 * j + 2 * tq;
        zr[2 * j] = (t0 + r0 < a.L) ? *reinterpret_cast<const uint32_t*>(zb + (size_t)r0 * a.ldp + p) : 0u;
        zr[2 * j + 1] = (t0 + r1 < a.L) ? *reinterpret_cast<const uint32_t*>(zb + (size_t)r1 * a.ldp + p) : 0u;
      }
    }
    ok = wait(&sm.mma2, i & 1) && ok;
    tc::fence_after_sync();
    // ---- I: gated output -> swizzled tile -> TMA store -----------------------------------------
    {
      float yo[16], pv[16];
      tc::tmem_ld_frag32(tmem + lane_base + TM_YOFF + 32 * half, yo);
      tc::tmem_ld_frag32(tmem + lane_base + TM_PV + 32 * half, pv);
      const float e0 = __expf(sm.cum[r0]), e1 = __expf(sm.cum[r1]);
      const float qd0 = Dh + (sm.qkp[0][r0] + sm.qkp[1][r0]) * sm.gam[r0];
      const float qd1 = Dh + (sm.qkp[0][r1] + sm.qkp[1][r1]) * sm.gam[r1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = 32 * half + 8 * j + 2 * tq;
        const float2 v0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.v + frag_off(r0, p)));
        const float2 v1 = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.v + frag_off(r1, p)));
        const float2 z0 = unpack_bf16(zr[2 * j]), z1 = unpack_bf16(zr[2 * j + 1]);
        const float a0 = (pv[4 * j] + e0 * yo[4 * j] + qd0 * v0.x) * z0.x * sigmoidf_(z0.x);
        const float a1 = (pv[4 * j + 1] + e0 * yo[4 * j + 1] + qd0 * v0.y) * z0.y * sigmoidf_(z0.y);
        const float a2 = (pv[4 * j + 2] + e1 * yo[4 * j + 2] + qd1 * v1.x) * z1.x * sigmoidf_(z1.x);
        const float a3 = (pv[4 * j + 3] + e1 * yo[4 * j + 3] + qd1 * v1.y) * z1.y * sigmoidf_(z1.y);
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r0, p)) = pack_bf16(a0, a1);
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r1, p)) = pack_bf16(a2, a3);
      }
    }
    if (tid < R) sm.th[tid] = sm.thnext[tid];
    tc::fence_proxy_async();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok);
    tc::fence_after_sync();
    if (tid == 0) {
      tc::tma_store_3d(&tm_y, h * P, t0, b, sm.p);
      tc::bulk_commit();
      store_pending = true;
    }
    if (!ok) break;
  }
  // ---- final state and angle ----------------------------------------------------------------
  if (ok && a.fin) {
    tc::fence_after_sync();
    float v[32];
    tc::tmem_ld32(tmem + lane_base + TM_ST + 32 * half, v);
    const int n = 32 * q + lane;
#pragma unroll
    for (int j = 0; j < 32; ++j) a.fin[(slot * P + 32 * half + j) * N + n] = v[j];
  }
  if (ok && a.thf && tid < R) a.thf[slot * R + tid] = sm.th[tid];
  if (!ok && tid == 0) {
    // a wait gave up: let the copies this CTA started land (bounded) before its shared memory
    // goes away, then report
    const int lb = bc_loads - 1, lv = vs_loads - 1;
    wait(&sm.bc_full, lb & 1);
    wait(&sm.vs_full[lv & 1], (lv >> 1) & 1);
    if (lv >= 1) wait(&sm.vs_full[(lv - 1) & 1], ((lv - 1) >> 1) & 1);
    if (a.status) atomicExch(a.status, 1);
  }
  if (tid == 0 && store_pending) tc::bulk_wait_all();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TM_COLS);
}

// =============================================================================================
// Backward: the chunk walker in reverse.  The gradient dS of the state after a chunk is carried
// in tensor memory (an M=128 fp32 tile, lane = state row n, 64 columns p) from the last chunk
// to the first, so the per-chunk dstate contributions, their reverse state pass and the chunk
// backward become one pass.  16 warps: row block rb = warp & 3 (its TMEM lane quadrant) and
// column quarter cq = warp >> 2.
//
// Per chunk (c = nc-1 .. 0), after its loads landed (stage ring, issued one chunk ahead):
//   prologue  row scalars, angles (from the forward's chunk-start angle), dY0 = dy silu(z),
//             exp(cum) dY0, the dz factor, Q / K in place, w V
//   D         dS_out(c): TMEM -> bf16 image (its dot with S_out(c) = S_in(c+1) gives d cum_end),
//             carry *= exp(chunk decay)
//   MMA 1     S = Q K^T, Yoff = Q S_in^T, dP = dY0 V^T, KdS = K dS_out^T,
//             carry += Q^T (exp(cum) dY0)                                 [carry -> dS_out(c-1)]
//   epi A     P, dS = dP * decay (masked) -> bf16 tiles; d cum row / column sums
//   MMA 2a    PV = P V, dQ = (exp(cum) dY0) S_in + dS K, dK = (w V) dS_out + dS^T Q
//   epi B1    dz (and d cum from dY0 . Yoff); MMA 2b: PdY = P^T dY0
//   epi C     dQ / dK: inverse rotation, dtheta, dscale, gQ / gK tiles, bias column sums
//   epi B3    dV = w KdS + PdY + (D + gamma qk) dY0; d cum from V . (w KdS)
//   F         per-row outputs (dtheta suffix sums, d decay, d gamma, d scale); TMA stores of
//             dz, dV, gQ, gK
// =============================================================================================
constexpr int BNT = 512;
constexpr uint32_t TB_S = 0, TB_DP = 64, TB_DQ = 0, TB_YOFF = 128, TB_PDY = 128, TB_KDS = 192, TB_PV = 256,
                   TB_DK = 320, TB_CAR = 448, TB_COLS = 512;

struct __align__(1024) BStage {
  unsigned char bn[2 * BOX];     // Bn -> K -> gK
  unsigned char cn[2 * BOX];     // Cn -> Q -> gQ
  unsigned char sin_[2 * BOX];   // S_in image [n][p] (from the forward)
  unsigned char v[BOX];          // V [s][p]
  unsigned char z[BOX];          // z -> dz factor -> dz
  unsigned char dy[BOX];         // dy -> dtheta table (fp32 [64][32], xor-swizzled)
  float rate[CS * R];            // rates -> theta
  float dt[CS + 4], sig[CS + 4], adt[CS], th0[R];
};
struct __align__(1024) BSmem {
  BStage stage[2];
  unsigned char dy0[BOX];        // dY0 = dy * silu(z)
  unsigned char edy0[BOX];       // exp(cum) dY0
  unsigned char wv[BOX];         // w V -> dV
  unsigned char dso[2 * BOX];    // dS_out image [n][p]
  unsigned char p[BOX];          // P [l][s]
  unsigned char ds[BOX];         // dS [l][s]
  float cum[CS], gam[CS], scl[CS], dqk[CS], dcum[CS], dscl[CS];
  float qkp[2][CS];
  float seg[16 * 32], misc[16];
  float cb[N], bb[N];
  uint64_t full[2], mma1, mma2, mma3, edge;
  uint32_t tslot;
};
static_assert(sizeof(BSmem) + 1024 <= 232448, "backward shared memory exceeds 227 KB");

struct BwdArgs {
  const bf16 *proj, *bc, *dy;
  const float *dt, *adt, *sig, *rate;
  const float *Bb, *Cb, *D;
  const bf16* states;            // the forward's S_in images
  const float* theta0;           // the forward's chunk-start angles
  const float* ds_fin;           // [B, nh, nseg, P, N] gradient of each segment's final state, or null
  const float* s_fin;            // [B, nh, P, N] the final state (with ds_fin at the sequence end), or null
  float* ds0;                    // [B, nh, nseg, P, N] gradient of each segment's initial state, or null
  float *dthl, *dthtot, *dgam, *dscl, *dadt;
  float *dD, *dCb, *dBb;         // [B, nh, nseg], [B, nh, nseg, N] x2 (partial sums per segment)
  int* status;
  int B, L, nh, ldp, lds, nc;
  int cps, nseg, seg_lo, seg_hi;
};

__device__ __forceinline__ int dth_idx(int row, int r) { return row * R + (r ^ ((row & 7) << 2)); }

__device__ __forceinline__ void bwd_load_stage(BSmem& sm, const BwdArgs& a, const CUtensorMap* tm_bc,
                                               const CUtensorMap* tm_proj, const CUtensorMap* tm_dy, int b, int h,
                                               int c, int j, int lane) {
  BStage& st = sm.stage[j & 1];
  uint64_t* bar = &sm.full[j & 1];
  const int t0 = c * CS, bh = b * a.nh + h;
  if (lane == 0) {
    tc::mbar_expect_tx(bar, 9 * BOX);
#pragma unroll
    for (int k = 0; k < 4; ++k) tc::tma_load_3d((k < 2 ? st.bn : st.cn) + (k & 1) * BOX, tm_bc, 64 * k, t0, b, bar);
    tc::tma_load_3d(st.v, tm_proj, a.nh * P + h * P, t0, b, bar);
    tc::tma_load_3d(st.z, tm_proj, h * P, t0, b, bar);
    tc::tma_load_3d(st.dy, tm_dy, h * P, t0, b, bar);
    tc::bulk_load(st.sin_, a.states + ((size_t)bh * a.nc + c) * (N * P), 2 * BOX, bar);
  }
  const float* rate = a.rate + (size_t)b * a.L * R;
  for (int i = lane; i < CS * R / 4; i += 32) {
    const int r = i >> 3, q = i & 7, t = t0 + r;
    const bool ok = t < a.L;
    cp_async16(st.rate + r * R + q * 4, rate + (size_t)(ok ? t : 0) * R + q * 4, ok ? 16 : 0);
  }
  const size_t row = (size_t)bh * a.lds;
  for (int i = lane; i < 3 * (CS + 1); i += 32) {
    const int which = i / (CS + 1), k = i % (CS + 1), t = t0 + k;
    if (which == 2 && k == CS) continue;
    const bool ok = t < a.L;
    const float* src = which == 0 ? a.dt : which == 1 ? a.sig : a.adt;
    float* dst = which == 0 ? st.dt : which == 1 ? st.sig : st.adt;
    cp_async4(dst + k, src + row + (ok ? t : 0), ok ? 4 : 0);
  }
  if (lane < R / 4) cp_async16(st.th0 + 4 * lane, a.theta0 + ((size_t)bh * a.nc + c) * R + 4 * lane);
  tc::cp_async_mbar_arrive(bar);
}

__global__ void __launch_bounds__(BNT, 1)
    m3_bwd_tc_k(BwdArgs a, const __grid_constant__ CUtensorMap tm_bc, const __grid_constant__ CUtensorMap tm_proj,
                const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_dproj,
                const __grid_constant__ CUtensorMap tm_gq, const __grid_constant__ CUtensorMap tm_gk) {
  extern __shared__ unsigned char smem_raw[];
  BSmem& sm = *reinterpret_cast<BSmem*>(smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nsl = a.seg_hi - a.seg_lo;
  const int bh = blockIdx.x / nsl, seg = a.seg_lo + blockIdx.x % nsl, b = bh / a.nh, h = bh % a.nh;
  const size_t slot = (size_t)bh * a.nseg + seg;
  const int nc = a.nc, cb = seg * a.cps, ce = min(nc, cb + a.cps), nw = ce - cb;
  const int rb = warp & 3, cq = warp >> 2, g = lane >> 2, tq = lane & 3;
  const int r0 = 16 * rb + g, r1 = r0 + 8, c16 = cq * 16;

  if (warp == 0) tc::tmem_alloc(&sm.tslot, TB_COLS);
  if (tid == 0) {
    tc::mbar_init(&sm.full[0], 33);
    tc::mbar_init(&sm.full[1], 33);
    tc::mbar_init(&sm.mma1, 1);
    tc::mbar_init(&sm.mma2, 1);
    tc::mbar_init(&sm.mma3, 1);
    tc::mbar_init(&sm.edge, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < N; i += BNT) {
    sm.cb[i] = a.Cb[h * N + i];
    sm.bb[i] = a.Bb[h * N + i];
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tslot;
  const uint32_t lane_base = (uint32_t)(32 * rb) << 16;
  // Q / K build ownership: warps 0-7 the rotated box (columns 0-63), warps 8-15 the other
  const int bhalf = warp >> 3, bu = (warp & 7) * 32 + lane, bch = bu & 7;
  float cbr[8], bbr[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    cbr[j] = sm.cb[64 * bhalf + 8 * bch + j];
    bbr[j] = sm.bb[64 * bhalf + 8 * bch + j];
  }
  // carry initialisation: the final state's gradient, or nothing (the first MMA overwrites)
  const bool have_fin = a.ds_fin != nullptr;
  if (have_fin) {
    float v[16];
    const int n = 32 * rb + lane;
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = a.ds_fin[(slot * P + c16 + j) * N + n];
    tc::tmem_st16(tmem + lane_base + TB_CAR + c16, v);
    tc::tmem_wait_st();
  }
  if (warp == 0) bwd_load_stage(sm, a, &tm_bc, &tm_proj, &tm_dy, b, h, ce - 1, 0, lane);
  // a segment that ends before the sequence does: S_out of its last chunk is the next chunk's
  // S_in image, read for that chunk's d cum_end (into the second stage, free until chunk 2)
  const bool edge = ce < nc;
  if (edge && tid == 0) {
    tc::mbar_expect_tx(&sm.edge, 2 * BOX);
    tc::bulk_load(sm.stage[1].sin_, a.states + ((size_t)bh * nc + ce) * (N * P), 2 * BOX, &sm.edge);
  }
  const float Dh = a.D[h];
  float colq[4][2], colk[4][2], dDacc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) colq[i][0] = colq[i][1] = colk[i][0] = colk[i][1] = 0.f;
  bool ok = true, store_pending = false;
  int loads = 1;

  for (int j = 0; j < nw; ++j) {
    const int c = ce - 1 - j, t0 = c * CS;
    BStage& st = sm.stage[j & 1];
    if (tid == 0 && store_pending) tc::bulk_wait_read();    // last chunk's stores have read their tiles
    if (tid < CS) {
      sm.dcum[tid] = 0.f;
      sm.dscl[tid] = 0.f;
    }
    __syncthreads();
    ok = wait(&sm.full[j & 1], (j >> 1) & 1) && ok;
    // ---- prologue: scalars and angles ------------------------------------------------------
    if (tid < CS) {
      const float d0 = st.dt[tid], s0_ = st.sig[tid], d1 = st.dt[tid + 1], s1 = st.sig[tid + 1];
      const float gm = d0 * s0_;
      sm.gam[tid] = gm;
      sm.scl[tid] = gm + d1 * (1.f - s1);
      float v = st.adt[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      sm.cum[tid] = v;
    }
    {   // theta prefix: thread (r = lane, seg = warp) owns rows 4*seg .. 4*seg+3
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = warp * 4 + i;
        acc += st.rate[row * R + lane] * st.dt[row];
        st.rate[th_idx(row, lane)] = acc;
      }
      sm.seg[warp * 32 + lane] = acc;
    }
    __syncthreads();
    if (tid >= 32 && tid < CS) sm.cum[tid] += sm.cum[31];
    {
      float base = st.th0[lane];
      for (int s2 = 0; s2 < warp; ++s2) base += sm.seg[s2 * 32 + lane];
#pragma unroll
      for (int i = 0; i < 4; ++i) st.rate[th_idx(warp * 4 + i, lane)] += base;
    }
    __syncthreads();
    const float cend = sm.cum[CS - 1];
    // ---- prologue: dY0, exp(cum) dY0, dz factor, dqk; Q / K in place; w V -------------------
    {
      const int row = tid >> 3, ch = tid & 7;
      const uint32_t off = swz(row, ch);
      const uint4 dv = *reinterpret_cast<const uint4*>(st.dy + off);
      const uint4 zv = *reinterpret_cast<const uint4*>(st.z + off);
      const uint4 xv = *reinterpret_cast<const uint4*>(st.v + off);
      const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w},
                     xw[4] = {xv.x, xv.y, xv.z, xv.w};
      const float e = __expf(sm.cum[row]), wr = __expf(cend - sm.cum[row]);
      uint32_t o0[4], o1[4], o2[4], o3[4];
      float dq = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 d2 = unpack_bf16(dw[k]), z2 = unpack_bf16(zw[k]), x2 = unpack_bf16(xw[k]);
        const float sg0 = sigmoidf_(z2.x), sg1 = sigmoidf_(z2.y);
        const float a0 = d2.x * z2.x * sg0, a1 = d2.y * z2.y * sg1;
        dq += a0 * x2.x + a1 * x2.y;
        o0[k] = pack_bf16(a0, a1);
        o1[k] = pack_bf16(a0 * e, a1 * e);
        o2[k] = pack_bf16(d2.x * sg0 * (1.f + z2.x * (1.f - sg0)), d2.y * sg1 * (1.f + z2.y * (1.f - sg1)));
        o3[k] = pack_bf16(x2.x * wr, x2.y * wr);
      }
      *reinterpret_cast<uint4*>(sm.dy0 + off) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
      *reinterpret_cast<uint4*>(sm.edy0 + off) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
      *reinterpret_cast<uint4*>(st.z + off) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
      *reinterpret_cast<uint4*>(sm.wv + off) = make_uint4(o3[0], o3[1], o3[2], o3[3]);
      dq += __shfl_xor_sync(0xffffffffu, dq, 1);
      dq += __shfl_xor_sync(0xffffffffu, dq, 2);
      dq += __shfl_xor_sync(0xffffffffu, dq, 4);
      if (ch == 0) sm.dqk[row] = dq;
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int row = (bu >> 3) + 32 * k;
      const uint32_t off = (uint32_t)bhalf * BOX + swz(row, bch);
      uint4* qp = reinterpret_cast<uint4*>(st.cn + off);
      uint4* kp = reinterpret_cast<uint4*>(st.bn + off);
      const uint4 cv = *qp, bv = *kp;
      const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
      float cqv[8], bk[8], qk = 0.f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float2 c2 = unpack_bf16(cw[m]), b2 = unpack_bf16(bw[m]);
        cqv[2 * m] = c2.x + cbr[2 * m];
        cqv[2 * m + 1] = c2.y + cbr[2 * m + 1];
        bk[2 * m] = b2.x + bbr[2 * m];
        bk[2 * m + 1] = b2.y + bbr[2 * m + 1];
        qk += cqv[2 * m] * bk[2 * m] + cqv[2 * m + 1] * bk[2 * m + 1];
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) qk += __shfl_xor_sync(0xffffffffu, qk, o);
      if (bch == 0) sm.qkp[bhalf][row] = qk;
      if (bhalf == 0) {
        const float4 th4 = *reinterpret_cast<const float4*>(st.rate + th_idx(row, 4 * bch));
        const float ths[4] = {th4.x, th4.y, th4.z, th4.w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float sn, cs;
          __sincosf(ths[m] - TWO_PI_F * floorf(ths[m] * (1.f / TWO_PI_F) + 0.5f), &sn, &cs);
          const float c0 = cqv[2 * m], c1 = cqv[2 * m + 1], b0 = bk[2 * m], b1 = bk[2 * m + 1];
          cqv[2 * m] = c0 * cs - c1 * sn;
          cqv[2 * m + 1] = c0 * sn + c1 * cs;
          bk[2 * m] = b0 * cs - b1 * sn;
          bk[2 * m + 1] = b0 * sn + b1 * cs;
        }
      }
      const float sc = sm.scl[row];
      *qp = make_uint4(pack_bf16(cqv[0], cqv[1]), pack_bf16(cqv[2], cqv[3]), pack_bf16(cqv[4], cqv[5]),
                       pack_bf16(cqv[6], cqv[7]));
      *kp = make_uint4(pack_bf16(bk[0] * sc, bk[1] * sc), pack_bf16(bk[2] * sc, bk[3] * sc),
                       pack_bf16(bk[4] * sc, bk[5] * sc), pack_bf16(bk[6] * sc, bk[7] * sc));
    }
    // ---- D: dS_out(c) image, d cum_end, carry *= exp(chunk decay) -----------------------------
    {
      const int n = 32 * rb + lane;
      const bool have = j > 0 || have_fin;
      float v[16];
      if (have) {
        tc::fence_after_sync();
        tc::tmem_ld16(tmem + lane_base + TB_CAR + c16, v);
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 2; ++k)
        *reinterpret_cast<uint4*>(sm.dso + swz(n, 2 * cq + k)) =
            make_uint4(pack_bf16(v[8 * k], v[8 * k + 1]), pack_bf16(v[8 * k + 2], v[8 * k + 3]),
                       pack_bf16(v[8 * k + 4], v[8 * k + 5]), pack_bf16(v[8 * k + 6], v[8 * k + 7]));
      float dot = 0.f;
      if (j == 0 && edge) ok = wait(&sm.edge, 0) && ok;
      if (j == 0 && !edge && have_fin && a.s_fin) {   // S_out of the last chunk is the final state
#pragma unroll
        for (int k = 0; k < 16; ++k) dot += v[k] * a.s_fin[(slot * P + c16 + k) * N + n];
      }
      if (j > 0 || edge) {   // S_out(c) = S_in(c+1): the other stage holds its image
        const unsigned char* so = sm.stage[(j + 1) & 1].sin_;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint4 sv = *reinterpret_cast<const uint4*>(so + swz(n, 2 * cq + k));
          const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float2 f = unpack_bf16(sw[m]);
            dot += f.x * v[8 * k + 2 * m] + f.y * v[8 * k + 2 * m + 1];
          }
        }
      }
      dot = warp_sum(dot);
      if (lane == 0) sm.misc[warp] = dot;
      if (have) {
        const float e = __expf(cend);
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] *= e;
        tc::tmem_st16(tmem + lane_base + TB_CAR + c16, v);
        tc::tmem_wait_st();
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok);
    tc::fence_after_sync();
    if (!ok) break;
    // ---- MMA group 1; then the next chunk's loads into the other stage -----------------------
    if (tid == 0) {
      const uint32_t id64 = tc::idesc_bf16(64, 64);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t aq = tc::desc_sw128(st.cn + (ks >> 2) * BOX, ks & 3);
        const uint64_t ak = tc::desc_sw128(st.bn + (ks >> 2) * BOX, ks & 3);
        tc::mma_bf16(tmem + TB_S, aq, ak, id64, ks > 0);
        tc::mma_bf16(tmem + TB_YOFF, aq, tc::desc_mn_sw128(st.sin_ + ks * 2048, BOX), id64 | tc::IDESC_B_MN, ks > 0);
        tc::mma_bf16(tmem + TB_KDS, ak, tc::desc_mn_sw128(sm.dso + ks * 2048, BOX), id64 | tc::IDESC_B_MN, ks > 0);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem + TB_DP, tc::desc_sw128(sm.dy0, ks), tc::desc_sw128(st.v, ks), id64, ks > 0);
      const uint32_t id128 = tc::idesc_bf16(128, 64) | tc::IDESC_A_MN | tc::IDESC_B_MN;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem + TB_CAR, tc::desc_mn_sw128(st.cn + ks * 2048, BOX),
                     tc::desc_mn_sw128(sm.edy0 + ks * 2048, BOX), id128, ks > 0 || j > 0 || have_fin);
      tc::commit(&sm.mma1);
    }
    if (warp == 0 && c > cb) bwd_load_stage(sm, a, &tm_bc, &tm_proj, &tm_dy, b, h, c - 1, j + 1, lane);
    if (c > cb) loads = j + 2;
    // ---- epilogue A: P, dS, d cum -------------------------------------------------------------
    ok = wait(&sm.mma1, j & 1) && ok;
    tc::fence_after_sync();
    const float cum0 = sm.cum[r0], cum1 = sm.cum[r1];
    {
      float pa[8], da[8];
      tc::tmem_ld_frag16(tmem + lane_base + TB_S + c16, pa);
      tc::tmem_ld_frag16(tmem + lane_base + TB_DP + c16, da);
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int s0c = c16 + nt * 8 + 2 * tq;
        const float cs0 = sm.cum[s0c], cs1 = sm.cum[s0c + 1];
        const float f00 = (s0c < r0) ? __expf(cum0 - cs0) : 0.f;
        const float f01 = (s0c + 1 < r0) ? __expf(cum0 - cs1) : 0.f;
        const float f10 = (s0c < r1) ? __expf(cum1 - cs0) : 0.f;
        const float f11 = (s0c + 1 < r1) ? __expf(cum1 - cs1) : 0.f;
        const float p00 = pa[4 * nt] * f00, p01 = pa[4 * nt + 1] * f01;
        const float p10 = pa[4 * nt + 2] * f10, p11 = pa[4 * nt + 3] * f11;
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r0, s0c)) = pack_bf16(p00, p01);
        *reinterpret_cast<uint32_t*>(sm.p + frag_off(r1, s0c)) = pack_bf16(p10, p11);
        const float g00 = da[4 * nt] * p00, g01 = da[4 * nt + 1] * p01;
        const float g10 = da[4 * nt + 2] * p10, g11 = da[4 * nt + 3] * p11;
        rs0 += g00 + g01;
        rs1 += g10 + g11;
        float ca = g00 + g10, cb = g01 + g11;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          ca += __shfl_xor_sync(0xffffffffu, ca, o);
          cb += __shfl_xor_sync(0xffffffffu, cb, o);
        }
        if (g == 0) {
          atomicAdd(&sm.dcum[s0c], -ca);
          atomicAdd(&sm.dcum[s0c + 1], -cb);
        }
        *reinterpret_cast<uint32_t*>(sm.ds + frag_off(r0, s0c)) = pack_bf16(da[4 * nt] * f00, da[4 * nt + 1] * f01);
        *reinterpret_cast<uint32_t*>(sm.ds + frag_off(r1, s0c)) =
            pack_bf16(da[4 * nt + 2] * f10, da[4 * nt + 3] * f11);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      if (tq == 0) {
        atomicAdd(&sm.dcum[r0], rs0);
        atomicAdd(&sm.dcum[r1], rs1);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // ---- MMA group 2a: PV, dQ, dK ----------------------------------------------------------------
    if (tid == 0) {
      const uint32_t id64 = tc::idesc_bf16(64, 64), idn = tc::idesc_bf16(64, 128);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        tc::mma_bf16(tmem + TB_PV, tc::desc_sw128(sm.p, ks), tc::desc_mn_sw128(st.v + ks * 2048, BOX),
                     id64 | tc::IDESC_B_MN, ks > 0);
        tc::mma_bf16(tmem + TB_DQ, tc::desc_sw128(sm.edy0, ks), tc::desc_sw128(st.sin_, ks), idn, ks > 0);
        tc::mma_bf16(tmem + TB_DK, tc::desc_sw128(sm.wv, ks), tc::desc_sw128(sm.dso, ks), idn, ks > 0);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        tc::mma_bf16(tmem + TB_DQ, tc::desc_sw128(sm.ds, ks), tc::desc_mn_sw128(st.bn + ks * 2048, BOX),
                     idn | tc::IDESC_B_MN, true);
        tc::mma_bf16(tmem + TB_DK, tc::desc_mn_sw128(sm.ds + ks * 2048, BOX),
                     tc::desc_mn_sw128(st.cn + ks * 2048, BOX), idn | tc::IDESC_A_MN | tc::IDESC_B_MN, true);
      }
      tc::commit(&sm.mma2);
    }
    // raw B rows of this thread's dQ / dK positions (global, L2-resident), fetched while the
    // MMAs run
    uint32_t braw[8];
    {
      const bf16* bcg = a.bc + ((size_t)b * a.L + t0) * (2 * N);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int row = hr ? r1 : r0;
        const bool live = t0 + row < a.L;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int n = c16 + (nt >> 1) * 64 + (nt & 1) * 8 + 2 * tq;
          braw[hr * 4 + nt] = live ? __ldg(reinterpret_cast<const unsigned int*>(bcg + (size_t)row * 2 * N + n)) : 0u;
        }
      }
    }
    ok = wait(&sm.mma2, j & 1) && ok;
    tc::fence_after_sync();
    const float e0 = __expf(cum0), e1 = __expf(cum1);
    const float q0 = Dh + (sm.qkp[0][r0] + sm.qkp[1][r0]) * sm.gam[r0];
    const float q1 = Dh + (sm.qkp[0][r1] + sm.qkp[1][r1]) * sm.gam[r1];
    // ---- epilogue B1: dz, d cum from dY0 . Yoff ---------------------------------------------------
    {
      float yo[8], pv[8];
      tc::tmem_ld_frag16(tmem + lane_base + TB_YOFF + c16, yo);
      tc::tmem_ld_frag16(tmem + lane_base + TB_PV + c16, pv);
      float dc0 = 0.f, dc1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int p = c16 + nt * 8 + 2 * tq;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int row = hr ? r1 : r0;
          const float qd = hr ? q1 : q0, er = hr ? e1 : e0;
          const uint32_t off = frag_off(row, p);
          const float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.v + off));
          const float2 f = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.z + off));
          const float2 d0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sm.dy0 + off));
          const float yo0 = er * yo[4 * nt + 2 * hr], yo1 = er * yo[4 * nt + 2 * hr + 1];
          const float y00 = pv[4 * nt + 2 * hr] + yo0 + qd * v.x;
          const float y01 = pv[4 * nt + 2 * hr + 1] + yo1 + qd * v.y;
          if (hr) dc1 += d0.x * yo0 + d0.y * yo1; else dc0 += d0.x * yo0 + d0.y * yo1;
          *reinterpret_cast<uint32_t*>(st.z + off) = pack_bf16(f.x * y00, f.y * y01);
        }
      }
      dc0 += __shfl_xor_sync(0xffffffffu, dc0, 1);
      dc0 += __shfl_xor_sync(0xffffffffu, dc0, 2);
      dc1 += __shfl_xor_sync(0xffffffffu, dc1, 1);
      dc1 += __shfl_xor_sync(0xffffffffu, dc1, 2);
      if (tq == 0) {
        atomicAdd(&sm.dcum[r0], dc0);
        atomicAdd(&sm.dcum[r1], dc1);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {   // MMA group 2b: PdY = P^T dY0 (into the dead Yoff columns); dz out
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tmem + TB_PDY, tc::desc_mn_sw128(sm.p + ks * 2048, BOX),
                     tc::desc_mn_sw128(sm.dy0 + ks * 2048, BOX),
                     tc::idesc_bf16(64, 64) | tc::IDESC_A_MN | tc::IDESC_B_MN, ks > 0);
      tc::commit(&sm.mma3);
      tc::tma_store_3d(&tm_dproj, h * P, t0, b, st.z);
      tc::bulk_commit();
      store_pending = true;
    }
    // ---- epilogue C: dQ / dK --------------------------------------------------------------------
    {
      float qa[16], ka[16];
      tc::tmem_ld_frag16(tmem + lane_base + TB_DQ + c16, qa);
      tc::tmem_ld_frag16(tmem + lane_base + TB_DQ + 64 + c16, qa + 8);
      tc::tmem_ld_frag16(tmem + lane_base + TB_DK + c16, ka);
      tc::tmem_ld_frag16(tmem + lane_base + TB_DK + 64 + c16, ka + 8);
      float* dth = reinterpret_cast<float*>(st.dy);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int row = hr ? r1 : r0;
        const bool live = t0 + row < a.L;
        const float sc = sm.scl[row];
        const float gm = sm.gam[row] * sm.dqk[row];
        float dsc = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int n = c16 + (nt >> 1) * 64 + (nt & 1) * 8 + 2 * tq;
          const int fi = (nt >> 1) * 8 + (nt & 1) * 4 + 2 * hr;     // register of this pair
          const float g0 = qa[fi], g1 = qa[fi + 1], k0g = ka[fi], k1g = ka[fi + 1];
          const float2 bn = unpack_bf16(braw[hr * 4 + nt]);
          const float b0 = bn.x + sm.bb[n], b1 = bn.y + sm.bb[n + 1];
          const uint32_t off = frag_off(row, n);
          const float2 qv = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.cn + off));
          float dq0, dq1, dk0, dk1, cb0, cb1;
          if (nt < 2) {   // rotated columns
            const int r = n >> 1;
            const float th = st.rate[th_idx(row, r)];
            float sn, cs;
            __sincosf(th - TWO_PI_F * floorf(th * (1.f / TWO_PI_F) + 0.5f), &sn, &cs);
            dq0 = g0 * cs + g1 * sn;
            dq1 = -g0 * sn + g1 * cs;
            const float kr0 = b0 * cs - b1 * sn, kr1 = b0 * sn + b1 * cs;
            dsc += k0g * kr0 + k1g * kr1;
            const float h0 = k0g * sc, h1 = k1g * sc;
            dth[dth_idx(row, r)] = (-g0 * qv.y + g1 * qv.x) + (-h0 * kr1 + h1 * kr0);
            dk0 = h0 * cs + h1 * sn;
            dk1 = -h0 * sn + h1 * cs;
            cb0 = qv.x * cs + qv.y * sn;
            cb1 = -qv.x * sn + qv.y * cs;
          } else {
            dq0 = g0;
            dq1 = g1;
            dsc += k0g * b0 + k1g * b1;
            dk0 = k0g * sc;
            dk1 = k1g * sc;
            cb0 = qv.x;
            cb1 = qv.y;
          }
          dq0 += gm * b0;
          dq1 += gm * b1;
          dk0 += gm * cb0;
          dk1 += gm * cb1;
          if (!live) dq0 = dq1 = dk0 = dk1 = 0.f;
          *reinterpret_cast<uint32_t*>(st.cn + off) = pack_bf16(dq0, dq1);
          *reinterpret_cast<uint32_t*>(st.bn + off) = pack_bf16(dk0, dk1);
          colq[nt][0] += dq0;
          colq[nt][1] += dq1;
          colk[nt][0] += dk0;
          colk[nt][1] += dk1;
        }
        dsc += __shfl_xor_sync(0xffffffffu, dsc, 1);
        dsc += __shfl_xor_sync(0xffffffffu, dsc, 2);
        if (tq == 0) atomicAdd(&sm.dscl[row], dsc);
      }
    }
    // ---- epilogue B3: dV ------------------------------------------------------------------------
    ok = wait(&sm.mma3, j & 1) && ok;
    tc::fence_after_sync();
    {
      float kd[8], pd[8];
      tc::tmem_ld_frag16(tmem + lane_base + TB_KDS + c16, kd);
      tc::tmem_ld_frag16(tmem + lane_base + TB_PDY + c16, pd);
      const float w0 = __expf(cend - cum0), w1 = __expf(cend - cum1);
      float dcs0 = 0.f, dcs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int p = c16 + nt * 8 + 2 * tq;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int row = hr ? r1 : r0;
          const float wr = hr ? w1 : w0, qd = hr ? q1 : q0;
          const uint32_t off = frag_off(row, p);
          const float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(st.v + off));
          const float2 d0 = unpack_bf16(*reinterpret_cast<const uint32_t*>(sm.dy0 + off));
          const float k0 = kd[4 * nt + 2 * hr] * wr, k1 = kd[4 * nt + 2 * hr + 1] * wr;
          if (hr) dcs1 += v.x * k0 + v.y * k1; else dcs0 += v.x * k0 + v.y * k1;
          *reinterpret_cast<uint32_t*>(sm.wv + off) =
              pack_bf16(k0 + pd[4 * nt + 2 * hr] + qd * d0.x, k1 + pd[4 * nt + 2 * hr + 1] + qd * d0.y);
        }
      }
      dcs0 += __shfl_xor_sync(0xffffffffu, dcs0, 1);
      dcs0 += __shfl_xor_sync(0xffffffffu, dcs0, 2);
      dcs1 += __shfl_xor_sync(0xffffffffu, dcs1, 1);
      dcs1 += __shfl_xor_sync(0xffffffffu, dcs1, 2);
      if (tq == 0) {
        atomicAdd(&sm.dcum[r0], -dcs0);
        atomicAdd(&sm.dcum[r1], -dcs1);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    ok = __syncthreads_and(ok);
    tc::fence_after_sync();
    // ---- F: stores and per-row outputs ------------------------------------------------------
    if (tid == 0) {
      tc::tma_store_3d(&tm_dproj, a.nh * P + h * P, t0, b, sm.wv);
      tc::tma_store_3d(&tm_gq, h * N, t0, b, st.cn);
      tc::tma_store_3d(&tm_gq, h * N + 64, t0, b, st.cn + BOX);
      tc::tma_store_3d(&tm_gk, h * N, t0, b, st.bn);
      tc::tma_store_3d(&tm_gk, h * N + 64, t0, b, st.bn + BOX);
      tc::bulk_commit();
      float dot = 0.f;
      for (int k = 0; k < BNT / 32; ++k) dot += sm.misc[k];
      sm.dcum[CS - 1] += dot;
    }
    if (tid < CS) dDacc += sm.dqk[tid];
    {   // dtheta suffix sums inside the chunk: thread (r = lane, seg = warp) owns rows 4*seg..+3
      const float* dth = reinterpret_cast<const float*>(st.dy);
      float acc = 0.f;
      float loc[4];
#pragma unroll
      for (int i = 3; i >= 0; --i) {
        acc += dth[dth_idx(warp * 4 + i, lane)];
        loc[i] = acc;
      }
      sm.seg[warp * 32 + lane] = acc;
      __syncthreads();
      float base = 0.f;
      for (int s2 = warp + 1; s2 < BNT / 32; ++s2) base += sm.seg[s2 * 32 + lane];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = warp * 4 + i, tt = t0 + row;
        const float G = base + loc[i];
        if (tt < a.L) a.dthl[(((size_t)b * a.L + tt) * a.nh + h) * R + lane] = G;
        if (row == 0) a.dthtot[((size_t)bh * nc + c) * R + lane] = G;
      }
    }
    if (tid < CS) {   // d decay: reverse inclusive scan of d cum inside the chunk
      float v = sm.dcum[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += u;
      }
      sm.cum[tid] = v;   // cum is dead: reuse it for the scan
    }
    __syncthreads();
    if (tid < CS) {
      const float v = sm.cum[tid] + (tid < 32 ? sm.cum[32] : 0.f);
      const int tt = t0 + tid;
      if (tt < a.L) {
        const size_t k = (size_t)bh * a.L + tt;
        a.dadt[k] = v;
        a.dgam[k] = sm.dqk[tid] * (sm.qkp[0][tid] + sm.qkp[1][tid]) + sm.dscl[tid];
        a.dscl[k] = sm.dscl[tid];
      }
    }
    store_pending = true;
  }
  // ---- end of the sequence: dS_in(0), dD, bias gradients -------------------------------------------
  if (ok && a.ds0) {
    tc::fence_after_sync();
    float v[16];
    tc::tmem_ld16(tmem + lane_base + TB_CAR + c16, v);
    const int n = 32 * rb + lane;
#pragma unroll
    for (int k = 0; k < 16; ++k) a.ds0[(slot * P + c16 + k) * N + n] = v[k];
  }
  __syncthreads();
  float* colsum = sm.seg;   // [2][N] (dead scratch)
  if (tid < 2 * N) colsum[tid] = 0.f;
  if (tid < 16) sm.misc[tid] = 0.f;
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int n = c16 + (nt >> 1) * 64 + (nt & 1) * 8 + 2 * tq;
    float a0 = colq[nt][0], a1 = colq[nt][1], k0 = colk[nt][0], k1 = colk[nt][1];
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      a0 += __shfl_xor_sync(0xffffffffu, a0, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
      k0 += __shfl_xor_sync(0xffffffffu, k0, o);
      k1 += __shfl_xor_sync(0xffffffffu, k1, o);
    }
    if (g == 0) {
      atomicAdd(&colsum[n], a0);
      atomicAdd(&colsum[n + 1], a1);
      atomicAdd(&colsum[N + n], k0);
      atomicAdd(&colsum[N + n + 1], k1);
    }
  }
  if (tid < CS) {
    const float d = warp_sum(dDacc);
    if (lane == 0) atomicAdd(&sm.misc[0], d);
  }
  __syncthreads();
  if (ok) {
    if (tid < N) a.dCb[slot * N + tid] = colsum[tid];
    else if (tid < 2 * N) a.dBb[slot * N + tid - N] = colsum[tid];
    if (tid == 0) a.dD[slot] = sm.misc[0];
  }
  if (!ok && tid == 0) {
    const int l = loads - 1;
    wait(&sm.full[l & 1], (l >> 1) & 1);
    if (l >= 1) wait(&sm.full[(l - 1) & 1], ((l - 1) >> 1) & 1);
    if (edge) wait(&sm.edge, 0);
    if (a.status) atomicExch(a.status, 1);
  }
  if (tid == 0 && store_pending) tc::bulk_wait_all();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TB_COLS);
}

// 3-D tensor map over a [B, L, width] bf16 tensor with row stride `ld` elements: box 64 x 64
static int map3(CUtensorMap* m, const void* ptr, int width, int L, int B, long ld) {
  const cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)L, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * L};
  const cuuint32_t box[3] = {64, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const auto enc = s0::tensor_map_encoder();
  if (!enc) return -4;
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : -4;
}

}  // namespace m3tc
}  // namespace s0

int m3_fwd_tc_launch(const M3TcFwd& f, cudaStream_t st) {
  using namespace s0::m3tc;
  FwdArgs a;
  a.proj = reinterpret_cast<const bf16*>(f.proj);
  a.dt = f.dt; a.adt = f.adt; a.sig = f.sig; a.rate = f.rate;
  a.Bb = f.Bb; a.Cb = f.Cb; a.D = f.D;
  a.states = reinterpret_cast<bf16*>(f.states);
  a.theta0 = f.theta0; a.s0 = f.s0; a.th_in = f.th_in; a.fin = f.fin; a.thf = f.thf; a.status = f.status;
  a.B = f.B; a.L = f.L; a.nh = f.nh; a.ldp = f.ldp; a.lds = f.lds; a.nc = (f.L + CS - 1) / CS;
  a.nseg = f.nseg > 0 ? f.nseg : 1;
  a.cps = (a.nc + a.nseg - 1) / a.nseg;
  a.seg_lo = f.seg_lo;
  a.seg_hi = f.seg_hi > 0 ? f.seg_hi : a.nseg;
  if (f.B <= 0 || f.L <= 0 || a.seg_hi <= a.seg_lo) return 0;
  if ((a.nseg - 1) * a.cps >= a.nc) return -5;   // every segment must own at least one chunk
  if ((reinterpret_cast<uintptr_t>(f.proj) | reinterpret_cast<uintptr_t>(f.bc) | reinterpret_cast<uintptr_t>(f.y) |
       reinterpret_cast<uintptr_t>(f.rate) | reinterpret_cast<uintptr_t>(f.states)) % 16 || f.ldp % 8)
    return -3;
  CUtensorMap tm_bc, tm_proj, tm_y;
  if (map3(&tm_bc, f.bc, 2 * N, f.L, f.B, 2 * N) || map3(&tm_proj, f.proj, f.ldp, f.L, f.B, f.ldp) ||
      map3(&tm_y, f.y, f.nh * P, f.L, f.B, (long)f.nh * P))
    return -4;
  const int smem = (int)sizeof(Smem) + 1024;
  cudaFuncSetAttribute(m3_fwd_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  m3_fwd_tc_k<<<f.B * f.nh * (a.seg_hi - a.seg_lo), NT, smem, st>>>(a, tm_bc, tm_proj, tm_y);
  return (int)cudaGetLastError();
}

int m3_bwd_tc_launch(const M3TcBwd& f, cudaStream_t st) {
  using namespace s0::m3tc;
  BwdArgs a;
  a.proj = reinterpret_cast<const bf16*>(f.proj);
  a.bc = reinterpret_cast<const bf16*>(f.bc);
  a.dy = reinterpret_cast<const bf16*>(f.dy);
  a.dt = f.dt; a.adt = f.adt; a.sig = f.sig; a.rate = f.rate;
  a.Bb = f.Bb; a.Cb = f.Cb; a.D = f.D;
  a.states = reinterpret_cast<const bf16*>(f.states);
  a.theta0 = f.theta0; a.ds_fin = f.ds_fin; a.s_fin = f.s_fin; a.ds0 = f.ds0;
  a.dthl = f.dthl; a.dthtot = f.dthtot; a.dgam = f.dgam; a.dscl = f.dscl; a.dadt = f.dadt;
  a.dD = f.dD; a.dCb = f.dCb; a.dBb = f.dBb; a.status = f.status;
  a.B = f.B; a.L = f.L; a.nh = f.nh; a.ldp = f.ldp; a.lds = f.lds; a.nc = (f.L + CS - 1) / CS;
  a.nseg = f.nseg > 0 ? f.nseg : 1;
  a.cps = (a.nc + a.nseg - 1) / a.nseg;
  a.seg_lo = f.seg_lo;
  a.seg_hi = f.seg_hi > 0 ? f.seg_hi : a.nseg;
  if (f.B <= 0 || f.L <= 0 || a.seg_hi <= a.seg_lo) return 0;
  if ((a.nseg - 1) * a.cps >= a.nc) return -5;
  if ((reinterpret_cast<uintptr_t>(f.proj) | reinterpret_cast<uintptr_t>(f.bc) | reinterpret_cast<uintptr_t>(f.dy) |
       reinterpret_cast<uintptr_t>(f.rate) | reinterpret_cast<uintptr_t>(f.states) |
       reinterpret_cast<uintptr_t>(f.theta0) | reinterpret_cast<uintptr_t>(f.dproj) |
       reinterpret_cast<uintptr_t>(f.gQ) | reinterpret_cast<uintptr_t>(f.gK)) % 16 ||
      f.ldp % 8)
    return -3;
  CUtensorMap tm_bc, tm_proj, tm_dy, tm_dproj, tm_gq, tm_gk;
  if (map3(&tm_bc, f.bc, 2 * N, f.L, f.B, 2 * N) || map3(&tm_proj, f.proj, f.ldp, f.L, f.B, f.ldp) ||
      map3(&tm_dy, f.dy, f.nh * P, f.L, f.B, (long)f.nh * P) || map3(&tm_dproj, f.dproj, f.ldp, f.L, f.B, f.ldp) ||
      map3(&tm_gq, f.gQ, f.nh * N, f.L, f.B, (long)f.nh * N) || map3(&tm_gk, f.gK, f.nh * N, f.L, f.B, (long)f.nh * N))
    return -4;
  const int smem = (int)sizeof(BSmem) + 1024;
  cudaFuncSetAttribute(m3_bwd_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  m3_bwd_tc_k<<<f.B * f.nh * (a.seg_hi - a.seg_lo), BNT, smem, st>>>(a, tm_bc, tm_proj, tm_dy, tm_dproj, tm_gq, tm_gk);
  return (int)cudaGetLastError();
}
