// Batched limit-order-book matching engine for sm_100a: one warp per book.
//
// Same semantics as the reference array engine
// (src/matching_engine/jaxob/JaxOrderBookArrays.py:84-682) and as the CPU oracle
// sigma0_b200/engine/book.py: fixed-capacity sides of `n_orders` rows
// [price, qty, oid, tid, sec, ns] with -1 rows empty, price-time priority,
// trades written to the first free trade row (else the last row), eviction of
// the worst price level when a side is full, cancel lookups by id then by init
// id at the price (then, in modes 2/3, a random order at the price is NOT
// supported on device: those modes run on the CPU engine), type-4 messages
// flipped and immediate-or-cancel, and the reference's switch routing.
//
// A warp keeps both sides and the trade rows of its book in shared memory for
// the whole message stream; every search (best order, first free row, id
// lookup, L2 levels) is a 4-entries-per-lane scan plus a warp reduction.
#include "common.cuh"
#include "launchers.h"

namespace s0 {
namespace eng {

constexpr int MAXO = 128;   // rows per side held in shared memory (n_orders <= 128)
constexpr int MAXT = 128;   // trade rows
constexpr int WPB = 4;      // books (warps) per block
constexpr int MAXINT = 2147483647;

struct Cfg {
  int n_orders, n_trades, init_id, book_depth, cancel_mode, type4, check_fill;
};

struct WarpBook {
  int* a;   // asks [MAXO][6]
  int* b;   // bids [MAXO][6]
  int* t;   // trades [MAXT][8]
};

// smallest index i < n with pred(i) true, or -1
template <typename F>
__device__ __forceinline__ int first_index(int n, F pred) {
  int lane = threadIdx.x & 31;
  for (int base = 0; base < n; base += 32) {
    int i = base + lane;
    unsigned m = __ballot_sync(0xffffffffu, i < n && pred(i));
    if (m) return base + __ffs(m) - 1;
  }
  return -1;
}

// best order on a side.  bid side: max price, then min sec, min ns, min index.
// ask side: min price with -1 treated as MAXINT, same tie-breaks.
__device__ __forceinline__ int top_index(const int* s, int n, bool bid) {
  int lane = threadIdx.x & 31;
  // first pass: best price
  int best = bid ? INT_MIN : MAXINT;
  for (int i = lane; i < n; i += 32) {
    int p = s[i * 6];
    if (bid) best = max(best, p);
    else best = min(best, p == -1 ? MAXINT : p);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    int v = __shfl_xor_sync(0xffffffffu, best, o);
    best = bid ? max(best, v) : min(best, v);
  }
  // exact reference order: among rows at `best`, min sec; among those, min ns;
  // first index.  Done in three reductions for clarity.
  int msec = MAXINT;
  for (int i = lane; i < n; i += 32)
    if (s[i * 6] == best) msec = min(msec, s[i * 6 + 4]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) msec = min(msec, __shfl_xor_sync(0xffffffffu, msec, o));
  int mns = MAXINT;
  for (int i = lane; i < n; i += 32) {
    int sec = s[i * 6] == best ? s[i * 6 + 4] : MAXINT;
    if (sec == msec) mns = min(mns, s[i * 6] == best ? s[i * 6 + 5] : MAXINT);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mns = min(mns, __shfl_xor_sync(0xffffffffu, mns, o));
  return first_index(n, [&](int i) {
    int sec = s[i * 6] == best ? s[i * 6 + 4] : MAXINT;
    int ns = sec == msec ? (s[i * 6] == best ? s[i * 6 + 5] : MAXINT) : MAXINT;
    return ns == mns;
  });
}

__device__ __forceinline__ void remove_nonpositive(int* s, int n) {
  int lane = threadIdx.x & 31;
  for (int i = lane; i < n; i += 32)
    if (s[i * 6 + 1] <= 0)
      for (int c = 0; c < 6; ++c) s[i * 6 + c] = -1;
  __syncwarp();
}

// match incoming quantity against `side` (bid side if bid_side); returns remaining
__device__ int match_against(int* side, int* trades, const Cfg& cfg, bool bid_side, int qtm, int price, int oid,
                             int sec, int ns, int tid, int s) {
  int lane = threadIdx.x & 31;
  for (int guard = 0; guard < 4 * MAXO; ++guard) {
    int top = top_index(side, cfg.n_orders, bid_side);
    int p = top >= 0 ? side[top * 6] : -1;
    bool crosses = bid_side ? (p >= price) : (p <= price);
    if (!(top >= 0 && crosses && qtm > 0 && p != -1)) break;
    int q = side[top * 6 + 1];
    int newq = max(0, q - qtm);
    int ti = first_index(cfg.n_trades, [&](int i) { return trades[i * 8 + 4] == -1; });   // column 4, as the reference
    if (ti < 0) ti = cfg.n_trades - 1;
    if (lane == 0) {
      int* tr = trades + ti * 8;
      tr[0] = p;
      tr[1] = -s * (q - newq);
      tr[2] = side[top * 6 + 2];
      tr[3] = oid;
      tr[4] = sec;
      tr[5] = ns;
      tr[6] = side[top * 6 + 3];
      tr[7] = tid;
      side[top * 6 + 1] = newq;
    }
    qtm = qtm - q;
    __syncwarp();
    remove_nonpositive(side, cfg.n_orders);
  }
  return qtm;
}

__device__ void add_order(int* side, const Cfg& cfg, int price, int qty, int oid, int tid, int sec, int ns) {
  int lane = threadIdx.x & 31;
  int idx = first_index(cfg.n_orders, [&](int i) {
    const int* r = side + i * 6;
    return r[0] == -1 || r[1] == -1 || r[2] == -1 || r[3] == -1 || r[4] == -1 || r[5] == -1;
  });
  if (idx < 0) idx = cfg.n_orders - 1;
  if (lane == 0) {
    int* r = side + idx * 6;
    r[0] = price; r[1] = max(0, qty); r[2] = oid; r[3] = tid; r[4] = sec; r[5] = ns;
  }
  __syncwarp();
  remove_nonpositive(side, cfg.n_orders);
}

__device__ void evict_if_full(int* side, const Cfg& cfg, bool worst_is_min) {
  int lane = threadIdx.x & 31;
  bool full = true;
  int worst = worst_is_min ? MAXINT : INT_MIN;
  for (int i = lane; i < cfg.n_orders; i += 32) {
    int p = side[i * 6];
    full &= (p >= 0);
    worst = worst_is_min ? min(worst, p) : max(worst, p);
  }
  full = __all_sync(0xffffffffu, full);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    int v = __shfl_xor_sync(0xffffffffu, worst, o);
    worst = worst_is_min ? min(worst, v) : max(worst, v);
  }
  if (full)
    for (int i = lane; i < cfg.n_orders; i += 32)
      if (side[i * 6] == worst)
        for (int c = 0; c < 6; ++c) side[i * 6 + c] = -1;
  __syncwarp();
}

__device__ void cancel(int* side, const Cfg& cfg, int price, int qty, int oid) {
  int lane = threadIdx.x & 31;
  int idx = first_index(cfg.n_orders, [&](int i) { return side[i * 6 + 2] == oid; });
  if (idx < 0 && cfg.cancel_mode != 0) {
    idx = first_index(cfg.n_orders, [&](int i) {
      const int* r = side + i * 6;
      return r[0] == price && r[2] <= cfg.init_id && r[2] >= cfg.init_id - cfg.book_depth * 2 && r[1] >= qty;
    });
  }
  if (idx < 0) idx = cfg.n_orders - 1;   // the reference's .at[-1]
  if (lane == 0) side[idx * 6 + 1] -= qty;
  __syncwarp();
  remove_nonpositive(side, cfg.n_orders);
}

__device__ void limit(WarpBook& wb, const Cfg& cfg, bool is_bid, int t, int p, int q, int oid, int tid, int sec,
                      int ns, int s, int* tmp) {
  int lane = threadIdx.x & 31;
  int rem;
  int* own;
  bool worst_is_min;
  if (is_bid) {
    rem = match_against(wb.a, wb.t, cfg, false, q, p, oid, sec, ns, tid, s);
    if (cfg.type4 == 2) p = MAXINT;
    own = wb.b;
    worst_is_min = true;
  } else {
    if (cfg.type4 == 2) p = 0;
    rem = match_against(wb.b, wb.t, cfg, true, q, p, oid, sec, ns, tid, s);
    own = wb.a;
    worst_is_min = false;
  }
  if (cfg.check_fill) evict_if_full(own, cfg, worst_is_min);
  bool ioc = (cfg.type4 == 0 || cfg.type4 == 2) && t == 4;
  if (ioc) return;   // executions never rest: post-eviction side is kept
  add_order(own, cfg, p, rem, oid, tid, sec, ns);
  (void)tmp;
  (void)lane;
}

__device__ void process_msg(WarpBook& wb, const Cfg& cfg, const int* m, int* tmp) {
  int t = m[0], sr = m[1], q = m[2], p = m[3], oid = m[4], tid = m[5], sec = m[6], ns = m[7];
  int s = (t == 4) ? -sr : sr;
  if (s == 0 && t == 0) return;
  if (s == -1 && (t == 2 || t == 3)) cancel(wb.a, cfg, p, q, oid);
  else if (s == 1 && (t == 2 || t == 3)) cancel(wb.b, cfg, p, q, oid);
  else if (s == 1 && (t == 1 || t == 4)) limit(wb, cfg, true, t, p, q, oid, tid, sec, ns, s, tmp);
  else limit(wb, cfg, false, t, p, q, oid, tid, sec, ns, s, tmp);
}

__global__ void __launch_bounds__(32 * WPB)
    eng_process(int* __restrict__ asks, int* __restrict__ bids, int* __restrict__ trades,
                const int* __restrict__ msgs, int n_msgs, int n_books, Cfg cfg) {
  __shared__ int sA[WPB][MAXO * 6], sB[WPB][MAXO * 6], sT[WPB][MAXT * 8], sTmp[WPB][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int book = blockIdx.x * WPB + w;
  if (book >= n_books) return;
  const int no = cfg.n_orders * 6, nt = cfg.n_trades * 8;
  int* ga = asks + (size_t)book * no;
  int* gb = bids + (size_t)book * no;
  int* gt = trades + (size_t)book * nt;
  for (int i = lane; i < no; i += 32) { sA[w][i] = ga[i]; sB[w][i] = gb[i]; }
  for (int i = lane; i < nt; i += 32) sT[w][i] = gt[i];
  __syncwarp();
  WarpBook wb{sA[w], sB[w], sT[w]};
  for (int k = 0; k < n_msgs; ++k) {
    const int* m = msgs + ((size_t)book * n_msgs + k) * 8;
    int mm[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) mm[c] = m[c];
    process_msg(wb, cfg, mm, sTmp[w]);
    __syncwarp();
  }
  for (int i = lane; i < no; i += 32) { ga[i] = sA[w][i]; gb[i] = sB[w][i]; }
  for (int i = lane; i < nt; i += 32) gt[i] = sT[w][i];
}

// L2 levels of one book (a warp): [ask_p, ask_v, bid_p, bid_v] x levels, missing
// levels (MAXINT, 0) / (-MAXINT, 0).  Asks ascend (empty rows = MAXINT), bids
// descend (empty = -1).  Lane 0 writes `o`.
__device__ void l2_levels(const int* a, const int* b, int n, int levels, int* o) {
  const int lane = threadIdx.x & 31;
  int prev_a = INT_MIN, prev_b = MAXINT;
  for (int l = 0; l < levels; ++l) {
    int pa = MAXINT, pb = INT_MIN;
    for (int i = lane; i < n; i += 32) {
      int x = a[i * 6];
      x = (x == -1) ? MAXINT : x;
      if (x > prev_a) pa = min(pa, x);
      int y = b[i * 6];
      if (y < prev_b) pb = max(pb, y);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      pa = min(pa, __shfl_xor_sync(0xffffffffu, pa, s));
      pb = max(pb, __shfl_xor_sync(0xffffffffu, pb, s));
    }
    bool a_ok = (pa != MAXINT) && (prev_a != MAXINT);
    bool b_ok = (pb != INT_MIN) && (pb != -1) && (prev_b != -1);
    int va = 0, vb = 0;
    for (int i = lane; i < n; i += 32) {
      if (a_ok && a[i * 6] == pa) va += a[i * 6 + 1];
      if (b_ok && b[i * 6] == pb) vb += b[i * 6 + 1];
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      va += __shfl_xor_sync(0xffffffffu, va, s);
      vb += __shfl_xor_sync(0xffffffffu, vb, s);
    }
    if (lane == 0) {
      o[4 * l + 0] = a_ok ? pa : MAXINT;
      o[4 * l + 1] = a_ok ? max(va, 0) : 0;
      o[4 * l + 2] = b_ok ? pb : -MAXINT;
      o[4 * l + 3] = b_ok ? max(vb, 0) : 0;
    }
    prev_a = a_ok ? pa : MAXINT;
    prev_b = b_ok ? pb : -1;
  }
}

__global__ void __launch_bounds__(32 * WPB)
    eng_l2(const int* __restrict__ asks, const int* __restrict__ bids, int* __restrict__ out, int levels,
           int n_books, Cfg cfg) {
  const int w = threadIdx.x >> 5;
  const int book = blockIdx.x * WPB + w;
  if (book >= n_books) return;
  l2_levels(asks + (size_t)book * cfg.n_orders * 6, bids + (size_t)book * cfg.n_orders * 6, cfg.n_orders, levels,
            out + (size_t)book * 4 * levels);
}

// ---------------------------------------------------------------------------
// Generation step: decode the sampled message, resolve its order id, match it,
// and emit L2 + the next book image -- the per-message tail of the reference's
// _generate_msg (src/base_model/inference/generate.py:1008-1061, get_sim_msg
// :386-520, _get_new_mid_price :703, transform_L2_state via preproc.py:119).
// ---------------------------------------------------------------------------
constexpr int NA_V = -9999;
constexpr int NEG_RET = -999999999;

__device__ __forceinline__ int special_val(int t) {
  return t == 0 ? -10000 : t == 1 ? -20000 : t == 2 ? -9999 : -30000;
}
__device__ __forceinline__ bool is_special(int v) {
  return v == -10000 || v == -20000 || v == -9999 || v == -30000;
}
// token -> field value for a field whose values are base + [0, n); tokens of
// other fields clamp to the nearest end (the binary-search decode of the table)
__device__ __forceinline__ int dec(int t, int off, int n, int base) {
  if (t < 4) return special_val(t);
  return base + min(max(t - off, 0), n - 1);
}
__device__ __forceinline__ int floordiv(int a, int b) {
  int q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}
// base-1000 digits (most significant first) -> value; NA if any digit (or the sign) is special
__device__ __forceinline__ int combine(const int* d, int n, int sign) {
  int v = 0;
  bool sp = is_special(sign);
  for (int i = 0; i < n; ++i) {
    sp |= is_special(d[i]);
    v = v * 1000 + d[i];
  }
  return sp ? NA_V : v * sign;
}

__device__ int dec_price(const int* tk, const GenLayout& L, int pos) {
  int st = tk[pos];
  int sign = st < 4 ? special_val(st) : (min(max(st - L.sign_off, 0), 1) == 0 ? -1 : 1);
  int d[4];
  for (int i = 0; i < L.price_digits; ++i) d[i] = dec(tk[pos + 1 + i], L.price_off, 1000, 0);
  return combine(d, L.price_digits, sign);
}
__device__ int dec_size(const int* tk, const GenLayout& L, int pos) {
  if (!L.size_digits) return dec(tk[pos], L.size_off, L.size_n, 0);
  return dec(tk[pos], L.size_off, 100, 0) * 100 + dec(tk[pos + 1], L.size_off, 100, 0);
}

__global__ void __launch_bounds__(32 * WPB)
    gen_apply(int* __restrict__ asks, int* __restrict__ bids, int* __restrict__ trades,
              const int64_t* __restrict__ toks, GenLayout L, Cfg cfg, const int* __restrict__ new_oid,
              int* __restrict__ p_mid, const int* __restrict__ time_in, int* __restrict__ raw_out,
              int* __restrict__ msg_out, int* __restrict__ prov_out, int* __restrict__ l2_out,
              float* __restrict__ img_out, int img_stride, int n_books, int apply, const int* __restrict__ inj) {
  __shared__ int sA[WPB][MAXO * 6], sB[WPB][MAXO * 6], sT[WPB][MAXT * 8], sTmp[WPB][32];
  __shared__ int sL2[WPB][4 * 64];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int book = blockIdx.x * WPB + w;
  if (book >= n_books) return;
  const int no = cfg.n_orders * 6, nt = cfg.n_trades * 8;
  int* ga = asks + (size_t)book * no;
  int* gb = bids + (size_t)book * no;
  int* gt = trades + (size_t)book * nt;
  for (int i = lane; i < no; i += 32) { sA[w][i] = ga[i]; sB[w][i] = gb[i]; }
  if (apply)
    for (int i = lane; i < nt; i += 32) sT[w][i] = gt[i];
  __syncwarp();
  const int pm_old = p_mid[book];
  int ts, tns;
  if (apply) {
    int tk[32];
    const int64_t* trow = toks + (size_t)book * L.msg_len;
    for (int i = 0; i < L.msg_len; ++i) tk[i] = (int)trow[i];
    int et, dir;
    if (L.fused_ed) {
      int ed = dec(tk[L.ev_pos], L.ev_off, 8, 0);
      et = floordiv(ed, 2) + 1;
      dir = ed - 2 * floordiv(ed, 2);
    } else {
      et = dec(tk[L.ev_pos], L.ev_off, 4, 1);
      dir = dec(tk[L.dir_pos], L.dir_off, 2, 0);
    }
    const int price = dec_price(tk, L, L.p_pos);
    const int size = dec_size(tk, L, L.s_pos);
    int tv[9];
    for (int i = 0; i < 9; ++i) tv[i] = dec(tk[L.dt_pos + i], L.time_off, 1000, 0);
    const int dts = tv[0], dtns = combine(tv + 1, 3, 1);
    ts = combine(tv + 4, 2, 1);
    tns = combine(tv + 6, 3, 1);
    const int pref = dec_price(tk, L, L.pref_pos);
    const int sref = dec_size(tk, L, L.sref_pos);
    int rv[5];
    for (int i = 0; i < 5; ++i) rv[i] = dec(tk[L.tref_pos + i], L.time_off, 1000, 0);
    const int tsr = combine(rv, 2, 1), tnsr = combine(rv + 2, 3, 1);
    const int p_abs = pm_old + price * L.tick;
    const bool is_cd = (et == 2) || (et == 3);
    const int* side = (dir == 1) ? sB[w] : sA[w];
    // level 1: exact reference timestamp; level 2: closest time at the price
    int i1 = first_index(cfg.n_orders, [&](int i) { return side[i * 6 + 4] == tsr && side[i * 6 + 5] == tnsr; });
    int oid_l1 = i1 >= 0 ? side[i1 * 6 + 2] : NEG_RET;
    int best = MAXINT, bi = MAXO;
    for (int i = lane; i < cfg.n_orders; i += 32) {
      const int* r = side + i * 6;
      if (r[0] == p_abs && r[1] > 0) {
        int d = (r[4] - tsr) * 1000 + floordiv(r[5] - tnsr, 1000000);
        d = abs(d);
        if (d < best || (d == best && i < bi)) { best = d; bi = i; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      int ob = __shfl_xor_sync(0xffffffffu, best, o), oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob < best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    int oid_l2 = bi < MAXO ? side[bi * 6 + 2] : NEG_RET;
    int oid_ref = oid_l1 != NEG_RET ? oid_l1 : oid_l2;
    int oid = is_cd ? oid_ref : new_oid[0];
    int m[8] = {et, dir * 2 - 1, size, p_abs, oid, -88, ts, tns};
    // do(Q): replace the generated order by [type, side, qty, mid + offset ticks]
    const bool injected = inj != nullptr && inj[0] != 0;
    if (injected) {
      m[0] = inj[1];
      m[1] = inj[2] * 2 - 1;
      m[2] = inj[3];
      m[3] = pm_old + inj[4] * L.tick;
      m[4] = new_oid[0];
    }
    if (lane == 0) {
      int* ro = raw_out + (size_t)book * 14;
      ro[0] = oid; ro[1] = et; ro[2] = dir; ro[3] = p_abs; ro[4] = price; ro[5] = size;
      ro[6] = dts; ro[7] = dtns; ro[8] = ts; ro[9] = tns; ro[10] = pref; ro[11] = sref; ro[12] = tsr; ro[13] = tnsr;
      for (int c = 0; c < 8; ++c) msg_out[(size_t)book * 8 + c] = m[c];
      int res = !is_cd ? 0 : (oid_l1 != NEG_RET ? 1 : (oid_l2 != NEG_RET ? 2 : 3));
      bool disagree = is_cd && pref != NA_V && price != NA_V && price != pref;
      prov_out[book] = res + (disagree ? 8 : 0) + (injected ? 16 : 0);
    }
    __syncwarp();
    WarpBook wb{sA[w], sB[w], sT[w]};
    process_msg(wb, cfg, m, sTmp[w]);
    __syncwarp();
    for (int i = lane; i < no; i += 32) { ga[i] = sA[w][i]; gb[i] = sB[w][i]; }
    for (int i = lane; i < nt; i += 32) gt[i] = sT[w][i];
  } else {
    ts = time_in[book * 2];
    tns = time_in[book * 2 + 1];
  }
  // best quotes and the new mid (kept when a side is empty)
  int ba = MAXINT, bb = INT_MIN;
  for (int i = lane; i < cfg.n_orders; i += 32) {
    int x = sA[w][i * 6];
    ba = min(ba, x == -1 ? MAXINT : x);
    bb = max(bb, sB[w][i * 6]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ba = min(ba, __shfl_xor_sync(0xffffffffu, ba, o));
    bb = max(bb, __shfl_xor_sync(0xffffffffu, bb, o));
  }
  if (ba == MAXINT) ba = -1;
  int pm_new = (ba <= 0 || bb <= 0) ? pm_old : ((ba + bb) / 2 / L.tick) * L.tick;
  if (!apply) pm_new = pm_old;
  const int p_change = floordiv(pm_new - pm_old, L.tick);
  l2_levels(sA[w], sB[w], cfg.n_orders, L.l2_levels, sL2[w]);
  __syncwarp();
  for (int i = lane; i < 4 * L.l2_levels; i += 32) l2_out[(size_t)book * 4 * L.l2_levels + i] = sL2[w][i];
  // book image: [p_change, day fraction, second fraction, volumes by price slot]
  float* img = img_out + (size_t)book * img_stride;
  for (int i = lane; i < L.img_levels; i += 32) img[3 + i] = 0.f;
  __syncwarp();
  if (lane == 0) {
    if (apply) p_mid[book] = pm_new;
    img[0] = (float)p_change;
    img[1] = ((float)ts - 34200.f) / 23400.f;
    img[2] = (float)tns / 1e9f;
    const int* o = sL2[w];
    const int nl = min(2 * L.l2_levels, 40);   // the reference transforms book_l2[0:40]
    long long mid = (long long)ceil((double)((long long)o[0] + (long long)o[2]) / (2.0 * L.tick)) * L.tick;
    for (int j = 0; j < nl; ++j) {
      long long p = o[2 * j];
      long long idx = p - mid;
      idx = (idx >= 0 ? idx / L.tick : -((-idx + L.tick - 1) / L.tick)) + L.img_levels / 2;
      if (idx >= 0 && idx < 500 && idx < L.img_levels) {
        float v = (float)o[2 * j + 1];
        img[3 + idx] = (idx >= L.img_levels / 2 ? -v : v) / 1000.f;
      }
    }
  }
}

}  // namespace eng
}  // namespace s0

void eng_process_launch(int* asks, int* bids, int* trades, const int* msgs, int n_msgs, int n_books, int n_orders,
                        int n_trades, int init_id, int book_depth, int cancel_mode, int type4, int check_fill,
                        cudaStream_t st) {
  s0::eng::Cfg c{n_orders, n_trades, init_id, book_depth, cancel_mode, type4, check_fill};
  int blocks = (n_books + s0::eng::WPB - 1) / s0::eng::WPB;
  s0::eng::eng_process<<<blocks, 32 * s0::eng::WPB, 0, st>>>(asks, bids, trades, msgs, n_msgs, n_books, c);
}

void eng_l2_launch(const int* asks, const int* bids, int* out, int levels, int n_books, int n_orders,
                   cudaStream_t st) {
  s0::eng::Cfg c{n_orders, 0, 0, 0, 0, 0, 0};
  int blocks = (n_books + s0::eng::WPB - 1) / s0::eng::WPB;
  s0::eng::eng_l2<<<blocks, 32 * s0::eng::WPB, 0, st>>>(asks, bids, out, levels, n_books, c);
}

void gen_apply_launch(int* asks, int* bids, int* trades, const int64_t* toks, const GenLayout& L, int n_orders,
                      int n_trades, int init_id, int book_depth, int cancel_mode, int type4, int check_fill,
                      const int* new_oid, int* p_mid, const int* time_in, int* raw_out, int* msg_out, int* prov_out,
                      int* l2_out, float* img_out, int img_stride, int n_books, int apply, const int* inj,
                      cudaStream_t st) {
  s0::eng::Cfg c{n_orders, n_trades, init_id, book_depth, cancel_mode, type4, check_fill};
  int blocks = (n_books + s0::eng::WPB - 1) / s0::eng::WPB;
  s0::eng::gen_apply<<<blocks, 32 * s0::eng::WPB, 0, st>>>(asks, bids, trades, toks, L, c, new_oid, p_mid, time_in,
                                                            raw_out, msg_out, prov_out, l2_out, img_out, img_stride,
                                                            n_books, apply, inj);
}
