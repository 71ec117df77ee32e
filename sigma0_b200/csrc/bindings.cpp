// Python bindings of the sigma0_b200 CUDA extension (module sigma0_b200._C).
//
// Tensor checks, allocation and stream selection live here; the .cu files hold
// torch-free kernels and raw-pointer launchers (launchers.h).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "launchers.h"

namespace {

constexpr int M3_N = 128, M3_P = 64, M3_R = 32;

int num_sms(const at::Tensor& t) {
  return at::cuda::getDeviceProperties(t.device().index())->multiProcessorCount;
}
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void req(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " has the wrong dtype");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

M3Geo m3_geo(const at::Tensor& proj, int64_t B, int64_t L, int64_t nh) {
  req(proj, at::kBFloat16, "proj");
  TORCH_CHECK(proj.size(-1) % 8 == 0, "proj row stride must be a multiple of 8");
  TORCH_CHECK(proj.size(-1) >= 2 * nh * M3_P + 2 * M3_N + 3 * nh + M3_R, "proj too narrow for the layout");
  TORCH_CHECK(proj.numel() == B * L * proj.size(-1), "proj shape does not match B*L rows");
  M3Geo g;
  g.B = (int)B; g.L = (int)L; g.nh = (int)nh; g.ldp = (int)proj.size(-1);
  return g;
}

struct M3Pre {
  at::Tensor bc, dt, adt, sig, rate, aend, angtot, theta0;
};

M3Scan m3_scan(const at::Tensor& proj, const M3Pre& pre, const at::Tensor& Bb, const at::Tensor& Cb,
               const at::Tensor& D) {
  M3Scan s;
  s.proj = proj.data_ptr();
  s.bc = pre.bc.data_ptr();
  s.dt = pre.dt.data_ptr<float>();
  s.adt = pre.adt.data_ptr<float>();
  s.sig = pre.sig.data_ptr<float>();
  s.rate = pre.rate.data_ptr<float>();
  s.Bb = Bb.data_ptr<float>();
  s.Cb = Cb.data_ptr<float>();
  s.D = D.data_ptr<float>();
  s.theta0 = pre.theta0.defined() ? pre.theta0.data_ptr<float>() : nullptr;
  s.aend = pre.aend.defined() ? pre.aend.data_ptr<float>() : nullptr;
  return s;
}

// per-token prep + chunk totals + angle carry
M3Pre m3_prepare(const at::Tensor& proj, int64_t B, int64_t L, int64_t nh, const at::Tensor& wB,
                 const at::Tensor& wC, const at::Tensor& dt_bias, double A_floor, double eps, bool totals = true) {
  M3Geo g = m3_geo(proj, B, L, nh);
  TORCH_CHECK(nh <= 64, "at most 64 heads");
  auto f32 = proj.options().dtype(at::kFloat);
  int nc = m3_nchunks((int)L);
  M3Pre pre;
  pre.bc = at::empty({B * L, 2 * M3_N}, proj.options());
  pre.dt = at::empty({B, nh, L}, f32);
  pre.adt = at::empty({B, nh, L}, f32);
  pre.sig = at::empty({B, nh, L}, f32);
  pre.rate = at::empty({B * L, M3_R}, f32);
  m3_prep_fwd_launch(g, proj.data_ptr(), wB.data_ptr<float>(), wC.data_ptr<float>(), dt_bias.data_ptr<float>(),
                     (float)A_floor, (float)eps, pre.bc.data_ptr(), pre.dt.data_ptr<float>(), pre.adt.data_ptr<float>(),
                     pre.sig.data_ptr<float>(), pre.rate.data_ptr<float>(), stream());
  if (!totals) return pre;
  pre.aend = at::empty({B, nh, nc}, f32);
  pre.angtot = at::empty({B, nh, nc, M3_R}, f32);
  pre.theta0 = at::empty({B, nh, nc, M3_R}, f32);
  M3Scan s0 = m3_scan(proj, pre, dt_bias, dt_bias, dt_bias);
  m3_chunk_totals_launch(g, s0, pre.aend.data_ptr<float>(), pre.angtot.data_ptr<float>(),
                         pre.theta0.data_ptr<float>(), stream());
  return pre;
}

// status word of the tcgen05 SSD kernels on each device (1 once a bounded wait gave up)
at::Tensor m3_status(const at::Tensor& like) {
  static std::vector<at::Tensor> per_dev(64);
  const int d = like.device().index();
  if (!per_dev[d].defined()) per_dev[d] = at::zeros({1}, like.options().dtype(at::kInt));
  return per_dev[d];
}
// status word of the tcgen05 GEMM on each device (1 once a bounded wait gave up)
at::Tensor gemm_status(const at::Tensor& like) {
  static std::vector<at::Tensor> per_dev(64);
  const int d = like.device().index();
  if (!per_dev[d].defined()) per_dev[d] = at::zeros({1}, like.options().dtype(at::kInt));
  return per_dev[d];
}

// C (+)= A . B on the tcgen05 GEMM.  `a` is [M, K] (a_mn false) or [K, M] (a_mn true), `b` is
// [K, N] (b_mn true) or [N, K] (b_mn false), both bf16 with unit column stride.  out_mode 0
// returns a new bf16 [M, N]; 1 / 2 store / reduce-add fp32 into `out` (unit column stride; its
// shape may be smaller than [M, N]: the rows / columns beyond it are dropped).
at::Tensor gemm_tc(const at::Tensor& a, const at::Tensor& b, bool a_mn, bool b_mn, int64_t out_mode,
                   c10::optional<at::Tensor> out, int64_t split_k) {
  // operands may be row-strided views (a slice of a wider buffer); rows must be contiguous
  auto rows_ok = [](const at::Tensor& t, at::ScalarType dt, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == dt, name, " has the wrong dtype");
    TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, ": a 2-D tensor with unit column stride");
  };
  rows_ok(a, at::kBFloat16, "a");
  rows_ok(b, at::kBFloat16, "b");
  const int64_t M = a_mn ? a.size(1) : a.size(0), K = a_mn ? a.size(0) : a.size(1);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1), N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK(K == Kb, "gemm_tc: inner dimensions differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(M > 0 && N > 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
              "gemm_tc: dimensions out of range");
  TORCH_CHECK(split_k >= 0 && (split_k <= 1 || out_mode == 2), "gemm_tc: K splits need out_mode 2");
  TORCH_CHECK(out_mode >= 0 && out_mode <= 2, "gemm_tc: out_mode is 0, 1 or 2");
  // the tensor maps want 16-byte aligned bases and row pitches
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0,
              "gemm_tc: operand row pitches must be multiples of 16 bytes (8 bf16)");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "gemm_tc: operands must start on 16-byte boundaries");
  if (out_mode == 0) TORCH_CHECK(N % 8 == 0, "gemm_tc: bf16 output rows must be multiples of 16 bytes (N % 8)");
  if (out_mode != 0) {
    TORCH_CHECK(out.has_value(), "gemm_tc: fp32 modes write into `out`");
    TORCH_CHECK((out->stride(0) * 4) % 16 == 0 && reinterpret_cast<uintptr_t>(out->data_ptr()) % 16 == 0,
                "gemm_tc: out must start on a 16-byte boundary with a row pitch of a multiple of 4 floats");
  }
  at::Tensor c;
  if (out_mode == 0) {
    c = at::empty({M, N}, a.options());
  } else {
    TORCH_CHECK(out.has_value(), "gemm_tc: fp32 modes write into `out`");
    c = *out;
    rows_ok(c, at::kFloat, "out");
    TORCH_CHECK(c.size(0) <= M && c.size(1) <= N, "gemm_tc: out larger than the product");
  }
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.C = c.data_ptr();
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.ldc = c.stride(0);
  g.c_rows = (int)c.size(0);
  g.c_cols = (int)c.size(1);
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.out_mode = (int)out_mode;
  g.split_k = (int)split_k;
  g.status = gemm_status(a).data_ptr<int>();
  const int e = gemm_tc_launch(g, num_sms(a), stream());
  TORCH_CHECK(e == 0, "gemm_tc launch failed: ", e);
  return c;
}

// the GLU block's fused GEMM epilogue: o = x . W with g = gelu(o) (both bf16); W is the [K, N]
// kernel in bf16, N a multiple of 64.
std::vector<at::Tensor> gemm_gelu_fwd(const at::Tensor& x, const at::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm_gelu_fwd: bf16 CUDA operands");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && x.size(1) == w.size(0),
              "gemm_gelu_fwd: x [M, K], w [K, N] with unit column stride");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(1);
  TORCH_CHECK(N % 64 == 0 && (x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm_gelu_fwd: N % 64 and 16-byte aligned rows");
  auto o = at::empty({M, N}, x.options()), g = at::empty({M, N}, x.options());
  c10::cuda::CUDAGuard guard(x.device());
  GemmArgs a{};
  a.A = x.data_ptr();
  a.B = w.data_ptr();
  a.C = o.data_ptr();
  a.C2 = g.data_ptr();
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.lda = x.stride(0); a.ldb = w.stride(0); a.ldc = N; a.ldc2 = N;
  a.c_rows = (int)M; a.c_cols = (int)N;
  a.a_mn = 0; a.b_mn = 1; a.out_mode = 3; a.split_k = 1;
  a.status = gemm_status(x).data_ptr<int>();
  const int e = gemm_tc_launch(a, num_sms(x), stream());
  TORCH_CHECK(e == 0, "gemm_gelu_fwd launch failed: ", e);
  return {o, g};
}

// y = x . W with W's rank row blocks all-gathered inside the GEMM (FSDP's first projection):
// `wfull` is this GPU's [K, N] gathered buffer (filled by the kernel), `src` the address of
// every rank's [K / world, N] row block (peer addresses), `ready` every rank's shard-version
// flag (peer addresses), `counters` `world` zeroed ints on this GPU.
at::Tensor gemm_ag(const at::Tensor& x, const at::Tensor& wfull, std::vector<int64_t> src, std::vector<int64_t> ready,
                   const at::Tensor& counters, int64_t rank, int64_t seq, int64_t spin) {
  TORCH_CHECK(x.is_cuda() && wfull.is_cuda() && x.scalar_type() == at::kBFloat16 && wfull.scalar_type() == at::kBFloat16,
              "gemm_ag: bf16 CUDA operands");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && wfull.dim() == 2 && wfull.is_contiguous() && x.size(1) == wfull.size(0),
              "gemm_ag: x [M, K] with unit column stride, wfull contiguous [K, N]");
  const int64_t world = (int64_t)src.size();
  TORCH_CHECK(world >= 2 && world <= 8 && (int64_t)ready.size() == world && counters.numel() >= world &&
                  counters.scalar_type() == at::kInt,
              "gemm_ag: 2..8 ranks, one source, flag and counter each");
  const int64_t M = x.size(0), K = x.size(1), N = wfull.size(1);
  TORCH_CHECK(K % (world * 64) == 0 && (x.stride(0) * 2) % 16 == 0 && (N * 2) % 16 == 0 && N % 8 == 0,
              "gemm_ag: K a multiple of 64 x world, 16-byte rows");
  auto y = at::empty({M, N}, x.options());
  c10::cuda::CUDAGuard guard(x.device());
  counters.zero_();
  GemmArgs a{};
  a.A = x.data_ptr();
  a.B = wfull.data_ptr();
  a.C = y.data_ptr();
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.lda = x.stride(0); a.ldb = N; a.ldc = N;
  a.c_rows = (int)M; a.c_cols = (int)N;
  a.a_mn = 0; a.b_mn = 1; a.out_mode = 0; a.split_k = 1;
  a.status = gemm_status(x).data_ptr<int>();
  a.ag_world = (int)world; a.ag_rank = (int)rank; a.ag_rows = (int)(K / world); a.ag_seq = (int)seq;
  for (int64_t r = 0; r < world; ++r) {
    a.ag_src[r] = reinterpret_cast<const void*>(src[r]);
    a.ag_ready[r] = reinterpret_cast<const int*>(ready[r]);
  }
  a.ag_count = counters.data_ptr<int>();
  a.ag_spin = spin;
  const int e = gemm_tc_launch(a, num_sms(x), stream());
  TORCH_CHECK(e == 0, "gemm_ag launch failed: ", e);
  return y;
}

// SSD implementation: 1 the tcgen05 chunk walkers, 0 the chunk-parallel mma.sync kernels,
// -1 (default) by occupancy: the walkers run one CTA per (sequence, head) and the backward one CTA
// per SM, so they are used when the backward's waves of CTAs keep at least 3/4 of the SMs busy.
// Measured training steps on one B200: 128 pairs (1 wave) 162.9 vs 173.8 ms with the walkers,
// 256 pairs (2 waves) the walkers by 3%, 160 pairs (a second wave of 12 CTAs) 407.6 vs 397.8 ms
// for the chunk-parallel kernels, which also win for a single sequence (32 pairs).
int g_m3_tc = -1;
bool m3_walker(const at::Tensor& like, int64_t B, int64_t nh) {
  if (g_m3_tc >= 0) return g_m3_tc == 1;
  const int64_t pairs = B * nh, sms = num_sms(like);
  const int64_t waves = (pairs + sms - 1) / sms;
  return 4 * pairs >= 3 * waves * sms;
}

// Segments per sequence for the walkers: one CTA walks one (sequence, head, segment).  With
// fewer (sequence, head) pairs than CTA slots (two per SM forward, one backward) each sequence
// is cut into segments that are walked in parallel from a zero state; a second pass re-walks
// every segment but the first (forward) / last (backward) from its true carried state.
int m3_segments(const at::Tensor& like, int64_t B, int64_t nh, int nc, int per_sm) {
  const char* e = getenv("S0_M3_SEGMENTS");
  int64_t want = e ? atoi(e) : (int64_t)per_sm * num_sms(like) / std::max<int64_t>(1, B * nh);
  want = std::max<int64_t>(1, std::min<int64_t>(want, nc));
  if (want <= 1) return 1;
  const int cps = (int)((nc + want - 1) / want);
  return (nc + cps - 1) / cps;
}

// per-segment totals of the decay ADT: [B, nh, nseg]
at::Tensor m3_segment_decay(const at::Tensor& adt, int64_t B, int64_t nh, int64_t L, int nseg, int cps) {
  const int64_t span = (int64_t)cps * 64;
  auto a = at::constant_pad_nd(adt.view({B, nh, L}), {0, span * nseg - L});
  return a.view({B, nh, nseg, span}).sum(-1);
}

// y = ssd(proj); returns (y, states, final state, final angle[, prep...]).  With the walker the
// prep is (bc, dt, adt, sig, rate, theta0) and `states` holds the S_in images for the backward.
std::vector<at::Tensor> m3_fwd(at::Tensor proj, int64_t B, int64_t L, int64_t nh, at::Tensor wB, at::Tensor wC,
                               at::Tensor dt_bias, at::Tensor Bb, at::Tensor Cb, at::Tensor D, double A_floor,
                               double eps, bool want_final = false, bool return_prep = false,
                               c10::optional<at::Tensor> init_state = c10::nullopt,
                               c10::optional<at::Tensor> init_angle = c10::nullopt) {
  c10::cuda::CUDAGuard guard(proj.device());
  M3Geo g = m3_geo(proj, B, L, nh);
  // a sequence continued from a carried state / angle (context parallelism) runs the walker
  const bool carried = (init_state.has_value() && init_state->defined()) ||
                       (init_angle.has_value() && init_angle->defined());
  const bool walker = carried || m3_walker(proj, B, nh);
  M3Pre pre = m3_prepare(proj, B, L, nh, wB, wC, dt_bias, A_floor, eps, !walker);
  int nc = m3_nchunks((int)L);
  at::Tensor fin, thf;
  if (want_final) fin = at::empty({B, nh, M3_P, M3_N}, proj.options().dtype(at::kFloat));
  auto y = at::empty({B, L, nh * M3_P}, proj.options());
  if (walker) {
    if (want_final) thf = at::empty({B, nh, M3_R}, proj.options().dtype(at::kFloat));
    M3TcFwd f{};
    f.proj = proj.data_ptr(); f.bc = pre.bc.data_ptr();
    f.dt = pre.dt.data_ptr<float>(); f.adt = pre.adt.data_ptr<float>(); f.sig = pre.sig.data_ptr<float>();
    f.rate = pre.rate.data_ptr<float>();
    f.Bb = Bb.data_ptr<float>(); f.Cb = Cb.data_ptr<float>(); f.D = D.data_ptr<float>();
    f.y = y.data_ptr();
    f.fin = want_final ? fin.data_ptr<float>() : nullptr;
    f.thf = want_final ? thf.data_ptr<float>() : nullptr;
    f.status = m3_status(proj).data_ptr<int>();
    f.B = (int)B; f.L = (int)L; f.nh = (int)nh; f.ldp = g.ldp; f.lds = (int)L;
    at::Tensor states, theta0;
    if (return_prep) {   // the S_in images and chunk-start angles the backward walks back over
      states = at::empty({B, nh, nc, M3_N * M3_P}, proj.options());
      theta0 = at::empty({B, nh, nc, M3_R}, proj.options().dtype(at::kFloat));
      f.states = states.data_ptr();
      f.theta0 = theta0.data_ptr<float>();
    }
    if (carried) {
      if (init_state.has_value() && init_state->defined()) {
        req(*init_state, at::kFloat, "init_state");
        TORCH_CHECK(init_state->numel() == B * nh * M3_P * M3_N, "init_state must be [B, nh, P, N]");
        f.s0 = init_state->data_ptr<float>();
      }
      if (init_angle.has_value() && init_angle->defined()) {
        req(*init_angle, at::kFloat, "init_angle");
        TORCH_CHECK(init_angle->numel() == B * nh * M3_R, "init_angle must be [B, nh, R]");
        f.th_in = init_angle->data_ptr<float>();
      }
    }
    const int nseg = carried ? 1 : m3_segments(proj, B, nh, nc, 2);
    if (nseg == 1) {
      const int rc = m3_fwd_tc_launch(f, stream());
      TORCH_CHECK(rc == 0, "m3_fwd_tc launch failed (", rc, ")");
    } else {
      const int cps = (nc + nseg - 1) / nseg;
      auto f32 = proj.options().dtype(at::kFloat);
      // segment start angles from the chunk angle carries; segment decay totals
      M3Geo g2 = g;
      auto aend = at::empty({B, nh, nc}, f32), angtot = at::empty({B, nh, nc, M3_R}, f32);
      auto th0all = at::empty({B, nh, nc, M3_R}, f32);
      M3Scan s0s = m3_scan(proj, pre, dt_bias, dt_bias, dt_bias);
      m3_chunk_totals_launch(g2, s0s, aend.data_ptr<float>(), angtot.data_ptr<float>(), th0all.data_ptr<float>(),
                             stream());
      auto th_in = th0all.slice(2, 0, nc, cps).contiguous();                       // [B, nh, nseg, R]
      auto adec = aend.view({B, nh, nc});
      auto segA = at::constant_pad_nd(adec, {0, (int64_t)nseg * cps - nc}).view({B, nh, nseg, cps}).sum(-1);
      auto fseg = at::empty({B, nh, nseg, M3_P, M3_N}, f32);
      auto thseg = at::empty({B, nh, nseg, M3_R}, f32);
      f.nseg = nseg;
      f.th_in = th_in.data_ptr<float>();
      f.fin = fseg.data_ptr<float>();
      f.thf = thseg.data_ptr<float>();
      int rc = m3_fwd_tc_launch(f, stream());                                      // pass 1: zero starts
      TORCH_CHECK(rc == 0, "m3_fwd_tc launch failed (", rc, ")");
      auto s_in = at::zeros_like(fseg);
      for (int k = 1; k < nseg; ++k)
        s_in.select(2, k).copy_(segA.select(2, k - 1).exp().unsqueeze(-1).unsqueeze(-1) * s_in.select(2, k - 1) +
                                fseg.select(2, k - 1));
      f.s0 = s_in.data_ptr<float>();
      f.seg_lo = 1;
      rc = m3_fwd_tc_launch(f, stream());                                           // pass 2: true starts
      TORCH_CHECK(rc == 0, "m3_fwd_tc launch failed (", rc, ")");
      if (want_final) {
        fin.copy_(fseg.select(2, nseg - 1));
        thf.copy_(thseg.select(2, nseg - 1));
      }
    }
    if (return_prep) return {y, states, fin, thf, pre.bc, pre.dt, pre.adt, pre.sig, pre.rate, theta0};
    return {y, states, fin, thf};
  }
  auto states = at::empty({B, nh, nc, M3_P, M3_N}, proj.options());
  M3Scan s = m3_scan(proj, pre, Bb, Cb, D);
  m3_states_launch(g, s, states.data_ptr(), stream(), want_final ? fin.data_ptr<float>() : nullptr);
  m3_scan_launch(g, s, states.data_ptr(), y.data_ptr(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (want_final) {
    // angle after the last token: theta0 of the last chunk + that chunk's total, mod 2pi
    auto last = pre.theta0.select(2, nc - 1) + pre.angtot.select(2, nc - 1);
    thf = last - 2 * M_PI * at::floor(last / (2 * M_PI));
  }
  if (return_prep)   // the per-token prep and chunk carries, so the backward need not recompute them
    return {y, states, fin, thf, pre.bc, pre.dt, pre.adt, pre.sig, pre.rate, pre.aend, pre.theta0};
  return {y, states, fin, thf};
}

// backward through the tcgen05 chunk walker; saved: the forward's (states, [bc, dt, adt, sig, rate, theta0])
std::vector<at::Tensor> m3_bwd_tc(at::Tensor proj, at::Tensor dy, at::Tensor wB, at::Tensor wC, at::Tensor dt_bias,
                                  at::Tensor Bb, at::Tensor Cb, at::Tensor D, int64_t B, int64_t L, int64_t nh,
                                  double A_floor, double eps, c10::optional<at::Tensor> saved_states,
                                  c10::optional<std::vector<at::Tensor>> saved_prep,
                                  c10::optional<at::Tensor> d_final = c10::nullopt, bool want_d_init = false,
                                  c10::optional<at::Tensor> final_state = c10::nullopt) {
  const bool carried = (d_final.has_value() && d_final->defined()) || want_d_init;
  M3Geo g = m3_geo(proj, B, L, nh);
  const int nc = m3_nchunks((int)L);
  at::Tensor bc, dt, adt, sig, rate, theta0, states;
  if (saved_prep.has_value() && saved_prep->size() == 6 && saved_states.has_value() && saved_states->defined()) {
    const auto& v = *saved_prep;
    bc = v[0]; dt = v[1]; adt = v[2]; sig = v[3]; rate = v[4]; theta0 = v[5];
    states = *saved_states;
    req(bc, at::kBFloat16, "saved_prep bc");
    req(states, at::kBFloat16, "saved_states");
    TORCH_CHECK(bc.numel() == B * L * 2 * M3_N && dt.numel() == B * nh * L && theta0.numel() == B * nh * nc * M3_R &&
                    states.numel() == B * nh * nc * M3_N * M3_P,
                "saved forward tensors do not match this call");
  } else {   // recompute: the forward walker writes the images (its y is discarded)
    auto fw = m3_fwd(proj, B, L, nh, wB, wC, dt_bias, Bb, Cb, D, A_floor, eps, false, true);
    states = fw[1]; bc = fw[4]; dt = fw[5]; adt = fw[6]; sig = fw[7]; rate = fw[8]; theta0 = fw[9];
  }
  auto f32 = proj.options().dtype(at::kFloat);
  auto dproj = at::empty_like(proj);
  auto gQ = at::empty({B * L, nh, M3_N}, proj.options());
  auto gK = at::empty({B * L, nh, M3_N}, proj.options());
  auto dthl = at::empty({B * L, nh, M3_R}, f32);
  auto dthtot = at::empty({B, nh, nc, M3_R}, f32);
  auto dgam = at::empty({B, nh, L}, f32), dscl = at::empty({B, nh, L}, f32), dadt = at::empty({B, nh, L}, f32);
  const int nseg = carried ? 1 : m3_segments(proj, B, nh, nc, 1);
  auto dD = at::empty({B, nh, nseg}, f32), dCb = at::empty({B, nh, nseg, M3_N}, f32),
       dBb = at::empty({B, nh, nseg, M3_N}, f32);
  M3TcBwd f{};
  f.proj = proj.data_ptr(); f.bc = bc.data_ptr(); f.dy = dy.data_ptr();
  f.dt = dt.data_ptr<float>(); f.adt = adt.data_ptr<float>(); f.sig = sig.data_ptr<float>();
  f.rate = rate.data_ptr<float>();
  f.Bb = Bb.data_ptr<float>(); f.Cb = Cb.data_ptr<float>(); f.D = D.data_ptr<float>();
  f.states = states.data_ptr(); f.theta0 = theta0.data_ptr<float>();
  f.dproj = dproj.data_ptr(); f.gQ = gQ.data_ptr(); f.gK = gK.data_ptr();
  f.dthl = dthl.data_ptr<float>(); f.dthtot = dthtot.data_ptr<float>(); f.dgam = dgam.data_ptr<float>();
  f.dscl = dscl.data_ptr<float>(); f.dadt = dadt.data_ptr<float>();
  f.dD = dD.data_ptr<float>(); f.dCb = dCb.data_ptr<float>(); f.dBb = dBb.data_ptr<float>();
  f.status = m3_status(proj).data_ptr<int>();
  f.B = (int)B; f.L = (int)L; f.nh = (int)nh; f.ldp = g.ldp; f.lds = (int)L;
  f.nseg = nseg;
  at::Tensor dinit;
  if (d_final.has_value() && d_final->defined()) {
    req(*d_final, at::kFloat, "d_final");
    TORCH_CHECK(d_final->numel() == B * nh * M3_P * M3_N, "d_final must be [B, nh, P, N]");
    TORCH_CHECK(final_state.has_value() && final_state->defined(),
                "d_final needs the forward's final state (its decay gradient)");
    req(*final_state, at::kFloat, "final_state");
    TORCH_CHECK(final_state->numel() == B * nh * M3_P * M3_N, "final_state must be [B, nh, P, N]");
    f.ds_fin = d_final->data_ptr<float>();
    f.s_fin = final_state->data_ptr<float>();
  }
  if (want_d_init) {
    dinit = at::empty({B, nh, M3_P, M3_N}, f32);
    f.ds0 = dinit.data_ptr<float>();
  }
  if (nseg == 1) {
    const int rc = m3_bwd_tc_launch(f, stream());
    TORCH_CHECK(rc == 0, "m3_bwd_tc launch failed (", rc, ")");
  } else {
    const int cps = (nc + nseg - 1) / nseg;
    auto segA = m3_segment_decay(adt, B, nh, L, nseg, cps);
    auto ds0 = at::empty({B, nh, nseg, M3_P, M3_N}, f32);
    f.ds0 = ds0.data_ptr<float>();
    int rc = m3_bwd_tc_launch(f, stream());                                        // pass 1: zero ends
    TORCH_CHECK(rc == 0, "m3_bwd_tc launch failed (", rc, ")");
    auto dend = at::zeros_like(ds0);
    for (int k = nseg - 2; k >= 0; --k)
      dend.select(2, k).copy_(segA.select(2, k + 1).exp().unsqueeze(-1).unsqueeze(-1) * dend.select(2, k + 1) +
                              ds0.select(2, k + 1));
    f.ds_fin = dend.data_ptr<float>();
    f.ds0 = nullptr;
    f.seg_hi = nseg - 1;
    rc = m3_bwd_tc_launch(f, stream());                                             // pass 2: true ends
    TORCH_CHECK(rc == 0, "m3_bwd_tc launch failed (", rc, ")");
  }
  m3_rev_carry_launch(g, dthtot.data_ptr<float>(), stream());
  auto dwB = at::zeros({M3_N}, f32), dwC = at::zeros({M3_N}, f32), ddtb = at::zeros({nh}, f32);
  m3_prep_bwd_launch(g, proj.data_ptr(), wB.data_ptr<float>(), wC.data_ptr<float>(), dt_bias.data_ptr<float>(),
                     (float)A_floor, (float)eps, gQ.data_ptr(), gK.data_ptr(), dthl.data_ptr<float>(),
                     dthtot.data_ptr<float>(), dgam.data_ptr<float>(), dscl.data_ptr<float>(),
                     dadt.data_ptr<float>(), dproj.data_ptr(), dwB.data_ptr<float>(), dwC.data_ptr<float>(),
                     ddtb.data_ptr<float>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  std::vector<at::Tensor> out = {dproj, dwB, dwC, ddtb, dD.sum(at::IntArrayRef{0, 2}),
                                 dCb.sum(at::IntArrayRef{0, 2}), dBb.sum(at::IntArrayRef{0, 2})};
  if (want_d_init) {
    // the initial angle shifts every token's angle: its gradient is the whole-sequence dtheta sum
    auto dth0 = dthl.view({B, L, nh, M3_R}).select(1, 0) + dthtot.select(2, 0);
    out.push_back(dinit);
    out.push_back(dth0);
  }
  return out;
}

std::vector<at::Tensor> m3_bwd(at::Tensor proj, at::Tensor dy, at::Tensor wB, at::Tensor wC, at::Tensor dt_bias,
                               at::Tensor Bb, at::Tensor Cb, at::Tensor D, int64_t B, int64_t L, int64_t nh,
                               double A_floor, double eps, c10::optional<at::Tensor> saved_states,
                               c10::optional<std::vector<at::Tensor>> saved_prep,
                               c10::optional<at::Tensor> d_final = c10::nullopt, bool want_d_init = false,
                               c10::optional<at::Tensor> final_state = c10::nullopt) {
  c10::cuda::CUDAGuard guard(proj.device());
  M3Geo g = m3_geo(proj, B, L, nh);
  req(dy, at::kBFloat16, "dy");
  // the saved forward tensors say which implementation wrote them (6 prep tensors: the walker)
  const bool carried = (d_final.has_value() && d_final->defined()) || want_d_init;
  const bool walker = saved_prep.has_value() && saved_states.has_value() && saved_states->defined()
                          ? saved_prep->size() == 6
                          : (carried || m3_walker(proj, B, nh));
  TORCH_CHECK(walker || !carried, "a carried state gradient needs the walker's saved forward tensors");
  if (walker)
    return m3_bwd_tc(proj, dy, wB, wC, dt_bias, Bb, Cb, D, B, L, nh, A_floor, eps, saved_states, saved_prep, d_final,
                     want_d_init, final_state);
  M3Pre pre;
  if (saved_prep.has_value() && saved_prep->size() == 7) {   // (bc, dt, adt, sig, rate, aend, theta0) of m3_fwd
    const auto& v = *saved_prep;
    pre.bc = v[0]; pre.dt = v[1]; pre.adt = v[2]; pre.sig = v[3]; pre.rate = v[4]; pre.aend = v[5]; pre.theta0 = v[6];
    req(pre.bc, at::kBFloat16, "saved_prep bc");
    TORCH_CHECK(pre.bc.numel() == B * L * 2 * M3_N && pre.dt.numel() == B * nh * L &&
                    pre.theta0.numel() == B * nh * m3_nchunks((int)L) * M3_R,
                "saved_prep shapes do not match this call");
  } else {
    pre = m3_prepare(proj, B, L, nh, wB, wC, dt_bias, A_floor, eps);
  }
  int nc = m3_nchunks((int)L);
  M3Scan s = m3_scan(proj, pre, Bb, Cb, D);
  at::Tensor states;
  if (saved_states.has_value() && saved_states->defined()) {   // the forward's passed states: no recompute
    states = *saved_states;
    req(states, at::kBFloat16, "saved_states");
    TORCH_CHECK(states.numel() == B * nh * nc * M3_P * M3_N, "saved_states shape");
  } else {
    states = at::empty({B, nh, nc, M3_P, M3_N}, proj.options());
    m3_states_launch(g, s, states.data_ptr(), stream());
  }
  auto U = at::empty({B, nh, nc, M3_P, M3_N}, proj.options());
  m3_dstates_launch(g, s, dy.data_ptr(), U.data_ptr(), stream());
  auto f32 = proj.options().dtype(at::kFloat);
  auto dproj = at::empty_like(proj);
  auto gQ = at::empty({B * L, nh, M3_N}, proj.options());
  auto gK = at::empty({B * L, nh, M3_N}, proj.options());
  auto dthl = at::empty({B * L, nh, M3_R}, f32);
  auto dthtot = at::empty({B, nh, nc, M3_R}, f32);
  auto dgam = at::empty({B, nh, L}, f32), dscl = at::empty({B, nh, L}, f32), dadt = at::empty({B, nh, L}, f32);
  auto dD = at::empty({B, nh, nc}, f32), dCb = at::empty({B, nh, nc, M3_N}, f32),
       dBb = at::empty({B, nh, nc, M3_N}, f32);
  M3BwdOut o;
  o.dproj = dproj.data_ptr();
  o.gQ = gQ.data_ptr();
  o.gK = gK.data_ptr();
  o.dthl = dthl.data_ptr<float>();
  o.dthtot = dthtot.data_ptr<float>();
  o.dgam = dgam.data_ptr<float>();
  o.dscl = dscl.data_ptr<float>();
  o.dadt = dadt.data_ptr<float>();
  o.dD = dD.data_ptr<float>();
  o.dCb = dCb.data_ptr<float>();
  o.dBb = dBb.data_ptr<float>();
  m3_chunk_bwd_launch(g, s, dy.data_ptr(), states.data_ptr(), U.data_ptr(), o, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto dwB = at::zeros({M3_N}, f32), dwC = at::zeros({M3_N}, f32), ddtb = at::zeros({nh}, f32);
  m3_prep_bwd_launch(g, proj.data_ptr(), wB.data_ptr<float>(), wC.data_ptr<float>(), dt_bias.data_ptr<float>(),
                     (float)A_floor, (float)eps, gQ.data_ptr(), gK.data_ptr(), dthl.data_ptr<float>(),
                     dthtot.data_ptr<float>(), dgam.data_ptr<float>(), dscl.data_ptr<float>(),
                     dadt.data_ptr<float>(), dproj.data_ptr(), dwB.data_ptr<float>(), dwC.data_ptr<float>(),
                     ddtb.data_ptr<float>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dproj, dwB, dwC, ddtb, dD.sum(at::IntArrayRef{0, 2}), dCb.sum(at::IntArrayRef{0, 2}),
          dBb.sum(at::IntArrayRef{0, 2})};
}

// ---- row / elementwise ------------------------------------------------------------------
std::vector<at::Tensor> ln_fwd(at::Tensor x, at::Tensor w, at::Tensor b, double eps) {
  req(x, at::kFloat, "x");
  c10::cuda::CUDAGuard guard(x.device());
  int64_t D = x.size(-1), T = x.numel() / D;
  TORCH_CHECK(D <= 2048, "LayerNorm width above 2048 is not supported");
  auto y = at::empty(x.sizes(), x.options().dtype(at::kBFloat16));
  auto mean = at::empty({T}, x.options()), rstd = at::empty({T}, x.options());
  ln_fwd_launch(x.data_ptr<float>(), w.data_ptr<float>(), b.data_ptr<float>(), y.data_ptr(), mean.data_ptr<float>(),
                rstd.data_ptr<float>(), T, (int)D, (float)eps, num_sms(x), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, mean, rstd};
}

std::vector<at::Tensor> ln_bwd(at::Tensor dy, at::Tensor x, at::Tensor mean, at::Tensor rstd, at::Tensor w,
                               c10::optional<at::Tensor> dres) {
  req(dy, at::kBFloat16, "dy");
  req(x, at::kFloat, "x");
  c10::cuda::CUDAGuard guard(x.device());
  int64_t D = x.size(-1), T = x.numel() / D;
  TORCH_CHECK(D % 4 == 0 && D <= 2048, "LayerNorm width must be a multiple of 4, at most 2048");
  auto dx = at::empty_like(x);
  auto dw = at::empty({D}, x.options()), db = at::empty({D}, x.options());
  auto part = at::empty({std::max<int64_t>(col_blocks(T, num_sms(x)), num_sms(x)), 2, D}, x.options());
  const float* r = nullptr;
  if (dres.has_value() && dres->defined()) {
    req(*dres, at::kFloat, "dres");
    r = dres->data_ptr<float>();
  }
  if (D > 512 && D <= 1024 && T >= num_sms(x))
    ln_bwd_pipe_launch(dy.data_ptr(), x.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                       w.data_ptr<float>(), r, dx.data_ptr<float>(), dw.data_ptr<float>(), db.data_ptr<float>(),
                       part.data_ptr<float>(), T, (int)D, num_sms(x), stream());
  else ln_bwd_launch(dy.data_ptr(), x.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                w.data_ptr<float>(), r, dx.data_ptr<float>(), dw.data_ptr<float>(), db.data_ptr<float>(),
                part.data_ptr<float>(), T, (int)D, num_sms(x), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, dw, db};
}

std::vector<at::Tensor> rms_fwd(at::Tensor x, at::Tensor w, double eps) {
  req(x, at::kBFloat16, "x");
  c10::cuda::CUDAGuard guard(x.device());
  int64_t D = x.size(-1), T = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8192, "RMSNorm width must be a multiple of 8, at most 8192");
  if (reinterpret_cast<uintptr_t>(w.data_ptr()) % 16) w = w.clone();   // the kernel reads w as float4
  auto y = at::empty_like(x);
  auto rstd = at::empty({T}, x.options().dtype(at::kFloat));
  if (D > 2048)
    rms_fwd_wide_launch(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), T, (int)D,
                        (float)eps, num_sms(x), stream());
  else
    rms_fwd_launch(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), T, (int)D, (float)eps,
                   num_sms(x), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

std::vector<at::Tensor> rms_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd) {
  req(dy, at::kBFloat16, "dy");
  req(x, at::kBFloat16, "x");
  c10::cuda::CUDAGuard guard(x.device());
  int64_t D = x.size(-1), T = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8192, "RMSNorm width must be a multiple of 8, at most 8192");
  if (reinterpret_cast<uintptr_t>(w.data_ptr()) % 16) w = w.clone();   // the kernel reads w as float4
  auto dx = at::empty_like(x);
  auto dw = at::empty({D}, x.options().dtype(at::kFloat));
  if (D > 2048) {
    auto wpart = at::empty({(int64_t)rms_wide_blocks(T, num_sms(x)), D}, x.options().dtype(at::kFloat));
    rms_bwd_wide_launch(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                        dw.data_ptr<float>(), wpart.data_ptr<float>(), T, (int)D, num_sms(x), stream());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {dx, dw};
  }
  auto part = at::empty({std::max<int64_t>(col_blocks(T, num_sms(x)), num_sms(x)), D}, x.options().dtype(at::kFloat));
  if (D > 1024 && D <= 2048 && T >= num_sms(x))
    rms_bwd_pipe_launch(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                        dw.data_ptr<float>(), part.data_ptr<float>(), T, (int)D, num_sms(x), stream());
  else
    rms_bwd_launch(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                   dw.data_ptr<float>(), part.data_ptr<float>(), T, (int)D, num_sms(x), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, dw};
}

at::Tensor gelu_fwd(at::Tensor o) {
  req(o, at::kBFloat16, "o");
  TORCH_CHECK(o.numel() % 8 == 0, "numel must be a multiple of 8");
  c10::cuda::CUDAGuard guard(o.device());
  auto g = at::empty_like(o);
  gelu_fwd_launch(o.data_ptr(), g.data_ptr(), o.numel(), num_sms(o), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return g;
}

at::Tensor glu_res_fwd(at::Tensor x, at::Tensor g, at::Tensor h, at::Tensor b) {
  req(x, at::kFloat, "x");
  req(g, at::kBFloat16, "g");
  req(h, at::kBFloat16, "h");
  int64_t D = x.size(-1);
  TORCH_CHECK(D % 8 == 0, "width must be a multiple of 8");
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty_like(x);
  glu_res_fwd_launch(x.data_ptr<float>(), g.data_ptr(), h.data_ptr(), b.data_ptr<float>(), out.data_ptr<float>(),
                     x.numel(), (int)D, num_sms(x), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> glu_res_bwd(at::Tensor dout, at::Tensor g, at::Tensor h, at::Tensor b) {
  req(dout, at::kFloat, "dout");
  int64_t D = dout.size(-1), T = dout.numel() / D;
  c10::cuda::CUDAGuard guard(dout.device());
  auto dh = at::empty(dout.sizes(), dout.options().dtype(at::kBFloat16));
  TORCH_CHECK(D % 4 == 0 && D <= 2048, "GLU width must be a multiple of 4, at most 2048");
  if (reinterpret_cast<uintptr_t>(b.data_ptr()) % 16) b = b.clone();   // read as float4
  auto dgp = at::empty_like(dout);
  auto db = at::empty({D}, dout.options());
  auto part = at::empty({(int64_t)glu_bwd_blocks(T, num_sms(dout)), D}, dout.options());
  glu_res_bwd_launch(dout.data_ptr<float>(), g.data_ptr(), h.data_ptr(), b.data_ptr<float>(), dh.data_ptr(),
                     dgp.data_ptr<float>(), db.data_ptr<float>(), part.data_ptr<float>(), T, (int)D, num_sms(dout),
                     stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dh, dgp, db};
}

at::Tensor gelu_bwd(at::Tensor o, at::Tensor dgp, at::Tensor dgm) {
  req(o, at::kBFloat16, "o");
  req(dgp, at::kFloat, "dgp");
  req(dgm, at::kBFloat16, "dgm");
  c10::cuda::CUDAGuard guard(o.device());
  auto d = at::empty_like(o);
  gelu_bwd_launch(o.data_ptr(), dgp.data_ptr<float>(), dgm.data_ptr(), d.data_ptr(), o.numel(), num_sms(o),
                  stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return d;
}

// logits [T, ld] bf16 (first V columns used) is overwritten with w[row]*(softmax - onehot).
at::Tensor ce_fwd_bwd(at::Tensor logits, c10::optional<at::Tensor> bias, at::Tensor labels,
                      c10::optional<at::Tensor> wrow, int64_t V) {
  req(logits, at::kBFloat16, "logits");
  req(labels, at::kLong, "labels");
  c10::cuda::CUDAGuard guard(logits.device());
  int64_t T = logits.size(0), ld = logits.size(1);
  auto loss = at::empty({T}, logits.options().dtype(at::kFloat));
  const float* bp = (bias.has_value() && bias->defined()) ? bias->data_ptr<float>() : nullptr;
  const float* wp = (wrow.has_value() && wrow->defined()) ? wrow->data_ptr<float>() : nullptr;
  ce_launch(logits.data_ptr(), bp, labels.data_ptr<int64_t>(), wp, loss.data_ptr<float>(), T, (int)V, (int)ld,
            stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return loss;
}

void sumsq(at::Tensor g, at::Tensor out) {
  req(g, at::kFloat, "g");
  c10::cuda::CUDAGuard guard(g.device());
  sumsq_launch(g.data_ptr<float>(), g.numel(), out.data_ptr<float>(), num_sms(g), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adam(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> pb,
          c10::optional<at::Tensor> sumsq_t, double max_norm, at::Tensor lr, double b1, double b2, double eps,
          double wd, double bc1, double bc2) {
  req(p, at::kFloat, "p");
  req(g, at::kFloat, "g");
  c10::cuda::CUDAGuard guard(p.device());
  void* pbp = (pb.has_value() && pb->defined()) ? pb->data_ptr() : nullptr;
  const float* ss = (sumsq_t.has_value() && sumsq_t->defined()) ? sumsq_t->data_ptr<float>() : nullptr;
  adam_launch(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), pbp, p.numel(), ss,
              (float)max_norm, lr.data_ptr<float>(), (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1,
              (float)bc2, num_sms(p), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---- tensor-parallel fused GEMM + all-reduce ------------------------------------------------
int64_t tp_gemm_allreduce(at::Tensor A, at::Tensor Bt, std::vector<int64_t> recv, int64_t rows_own,
                          std::vector<int64_t> out, std::vector<int64_t> flags, int64_t rank, int64_t seq,
                          int64_t spin_limit, at::Tensor status, at::Tensor abort,
                          c10::optional<at::Tensor> stamps) {
  req(A, at::kBFloat16, "A");
  req(Bt, at::kBFloat16, "Bt");
  TORCH_CHECK(A.dim() == 2 && Bt.dim() == 2 && A.size(1) == Bt.size(1), "A [M, K] and Bt [N, K]");
  const int world = (int)recv.size();
  TORCH_CHECK(world >= 1 && world <= TPF_MAXW && (int)out.size() == world && (int)flags.size() == world,
              "one receive, output and flag pointer per rank (at most ", TPF_MAXW, ")");
  c10::cuda::CUDAGuard guard(A.device());
  TpfArgs a;
  a.A = reinterpret_cast<const __nv_bfloat16*>(A.data_ptr());
  a.Bt = reinterpret_cast<const __nv_bfloat16*>(Bt.data_ptr());
  a.M = (int)A.size(0); a.N = (int)Bt.size(0); a.K = (int)A.size(1);
  for (int k = 0; k < TPF_MAXW; ++k) {
    a.recv[k] = k < world ? reinterpret_cast<__nv_bfloat16*>(recv[k]) : nullptr;
    a.out[k] = k < world ? reinterpret_cast<__nv_bfloat16*>(out[k]) : nullptr;
    a.flags[k] = k < world ? reinterpret_cast<int*>(flags[k]) : nullptr;
  }
  a.world = world; a.rank = (int)rank; a.seq = (int)seq; a.spin_limit = spin_limit;
  a.rows_own = rows_own;
  TORCH_CHECK(rows_own * world >= (A.size(0) + 127) / 128 * 128 && rows_own % 128 == 0, "receive slots too small");
  a.status = status.data_ptr<int>();
  a.abort = abort.data_ptr<int>();
  a.stamps = nullptr;
  if (stamps && stamps->defined()) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->is_cuda() && stamps->numel() >= 4 + num_sms(A),
                "stamps: int64 CUDA tensor of at least 4 + SM-count entries");
    a.stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  return tp_gemm_allreduce_launch(a, num_sms(A), stream());
}

// ---- attention ----------------------------------------------------------------------------
static void attn_check(const at::Tensor& t, const char* name, int64_t hd) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a bf16 CUDA tensor");
  TORCH_CHECK(t.dim() == 4 && t.size(3) == hd && t.stride(3) == 1, name, ": [B, L, nh, ", hd, "] with a contiguous head dim");
  TORCH_CHECK(t.stride(0) % 8 == 0 && t.stride(1) % 8 == 0 && t.stride(2) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, ": strides must be multiples of 8 elements and the base 16-byte aligned");
}

static AttnArgs attn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                          const at::Tensor& lse, double scale, int64_t window, int64_t q_offset,
                          const c10::optional<at::Tensor>& kpos, const c10::optional<at::Tensor>& qoff) {
  const int64_t hd = q.size(3);
  TORCH_CHECK(hd == 64 || hd == 128, "attention head dim must be 64 or 128, got ", hd);
  attn_check(q, "q", hd);
  attn_check(k, "k", hd);
  attn_check(v, "v", hd);
  attn_check(o, "o", hd);
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(2) == k.size(2) && o.sizes() == q.sizes(),
              "q/o [B, Lq, nh, hd] and k/v [B, Lk, nh, hd]");
  req(lse, at::kFloat, "lse");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == q.size(0) * q.size(2) * q.size(1), "lse [B, nh, Lq]");
  AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.sq_b = q.stride(0); a.sq_l = q.stride(1); a.sq_h = q.stride(2);
  a.sk_b = k.stride(0); a.sk_l = k.stride(1); a.sk_h = k.stride(2);
  a.sv_b = v.stride(0); a.sv_l = v.stride(1); a.sv_h = v.stride(2);
  a.so_b = o.stride(0); a.so_l = o.stride(1); a.so_h = o.stride(2);
  a.B = (int)q.size(0); a.nh = (int)q.size(2); a.Lq = (int)q.size(1); a.Lk = (int)k.size(1);
  a.q_offset = (int)q_offset; a.window = (int)window;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.kpos = nullptr;
  a.qoff = nullptr;
  a.status = nullptr;
  a.kblk = nullptr;
  a.kb_n = 0; a.kb_ng = 1; a.kb_max = 0;
  if (kpos && kpos->defined()) {
    req(*kpos, at::kInt, "kpos");
    TORCH_CHECK(kpos->is_contiguous() && kpos->dim() == 2 && kpos->size(0) == k.size(0) && kpos->size(1) == k.size(1),
                "kpos [B, Lk] int32");
    a.kpos = kpos->data_ptr<int>();
  }
  if (qoff && qoff->defined()) {
    req(*qoff, at::kInt, "qoff");
    TORCH_CHECK(qoff->is_contiguous() && qoff->numel() == q.size(0), "qoff [B] int32");
    a.qoff = qoff->data_ptr<int>();
  }
  return a;
}

void attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, double scale, int64_t window,
              int64_t q_offset, c10::optional<at::Tensor> kpos, c10::optional<at::Tensor> qoff) {
  c10::cuda::CUDAGuard guard(q.device());
  const AttnArgs a = attn_args(q, k, v, o, lse, scale, window, q_offset, kpos, qoff);
  const int rc = attn_fwd_launch(a, (int)q.size(3), stream());
  TORCH_CHECK(rc == 0, "attn_fwd launch failed (", rc, ")");
}

void attn_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, at::Tensor dout, at::Tensor D,
              at::Tensor dq_acc, at::Tensor dk, at::Tensor dv, double scale, int64_t window, int64_t q_offset,
              c10::optional<at::Tensor> kpos, c10::optional<at::Tensor> qoff) {
  c10::cuda::CUDAGuard guard(q.device());
  AttnBwdArgs a;
  a.f = attn_args(q, k, v, o, lse, scale, window, q_offset, kpos, qoff);
  const int64_t hd = q.size(3);
  attn_check(dout, "dout", hd);
  attn_check(dk, "dk", hd);
  attn_check(dv, "dv", hd);
  TORCH_CHECK(dout.sizes() == q.sizes() && dk.sizes() == k.sizes() && dv.sizes() == v.sizes(), "gradient shapes");
  req(D, at::kFloat, "D");
  req(dq_acc, at::kFloat, "dq_acc");
  TORCH_CHECK(D.is_contiguous() && D.numel() == lse.numel(), "D [B, nh, Lq]");
  TORCH_CHECK(dq_acc.is_contiguous() && dq_acc.sizes() == q.sizes(), "dq_acc [B, Lq, nh, hd] fp32, contiguous");
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.sd_b = dout.stride(0); a.sd_l = dout.stride(1); a.sd_h = dout.stride(2);
  a.D = D.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.sdk_b = dk.stride(0); a.sdk_l = dk.stride(1); a.sdk_h = dk.stride(2);
  a.sdv_b = dv.stride(0); a.sdv_l = dv.stride(1); a.sdv_h = dv.stride(2);
  a.scale = (float)scale;
  a.dk_acc = a.dv_acc = nullptr;
  a.kb_lsrc = 0;
  const int rc = attn_bwd_launch(a, (int)hd, stream());
  TORCH_CHECK(rc == 0, "attn_bwd launch failed (", rc, ")");
}

// Block-indirect keys (NSA selected branch): entry e (query group) attends to the 64-key
// blocks kblk[e] of source batch e / (E / B) of k / v [B, Lsrc, nh, hd], so the selected
// blocks are never gathered; kpos [E, 64 kb_n] gives every logical key its absolute
// position, qoff [E] every entry its first query position.
static AttnArgs attn_sel_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                              const at::Tensor& lse, double scale, const at::Tensor& kblk, const at::Tensor& kpos,
                              const at::Tensor& qoff) {
  const int64_t hd = q.size(3);
  TORCH_CHECK(hd == 64 || hd == 128, "attention head dim must be 64 or 128, got ", hd);
  attn_check(q, "q", hd);
  attn_check(k, "k", hd);
  attn_check(v, "v", hd);
  attn_check(o, "o", hd);
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(2) == k.size(2) && o.sizes() == q.sizes(),
              "q/o [E, Lq, nh, hd] and k/v [B, Lsrc, nh, hd]");
  const int64_t E = q.size(0), Bs = k.size(0);
  TORCH_CHECK(Bs > 0 && E % Bs == 0, "entries must be a multiple of the source batch");
  TORCH_CHECK(k.size(1) >= 64, "the source must hold at least one 64-key block");
  req(kblk, at::kInt, "kblk");
  TORCH_CHECK(kblk.is_contiguous() && kblk.dim() == 2 && kblk.size(0) == E && kblk.size(1) > 0, "kblk [E, nblk] int32");
  const int64_t Lk = 64 * kblk.size(1);
  req(kpos, at::kInt, "kpos");
  TORCH_CHECK(kpos.is_contiguous() && kpos.dim() == 2 && kpos.size(0) == E && kpos.size(1) == Lk, "kpos [E, 64 nblk]");
  req(qoff, at::kInt, "qoff");
  TORCH_CHECK(qoff.is_contiguous() && qoff.numel() == E, "qoff [E] int32");
  req(lse, at::kFloat, "lse");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == E * q.size(2) * q.size(1), "lse [E, nh, Lq]");
  AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.sq_b = q.stride(0); a.sq_l = q.stride(1); a.sq_h = q.stride(2);
  a.sk_b = k.stride(0); a.sk_l = k.stride(1); a.sk_h = k.stride(2);
  a.sv_b = v.stride(0); a.sv_l = v.stride(1); a.sv_h = v.stride(2);
  a.so_b = o.stride(0); a.so_l = o.stride(1); a.so_h = o.stride(2);
  a.B = (int)E; a.nh = (int)q.size(2); a.Lq = (int)q.size(1); a.Lk = (int)Lk;
  a.q_offset = 0; a.window = 0;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.kpos = kpos.data_ptr<int>();
  a.qoff = qoff.data_ptr<int>();
  a.status = nullptr;
  a.kblk = kblk.data_ptr<int>();
  a.kb_n = (int)kblk.size(1); a.kb_ng = (int)(E / Bs); a.kb_max = (int)(k.size(1) / 64) - 1;
  return a;
}

void attn_sel_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, double scale,
                  at::Tensor kblk, at::Tensor kpos, at::Tensor qoff) {
  c10::cuda::CUDAGuard guard(q.device());
  const AttnArgs a = attn_sel_args(q, k, v, o, lse, scale, kblk, kpos, qoff);
  const int rc = attn_fwd_launch(a, (int)q.size(3), stream());
  TORCH_CHECK(rc == 0, "attn_sel_fwd launch failed (", rc, ")");
}

void attn_sel_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, at::Tensor dout,
                  at::Tensor D, at::Tensor dq_acc, at::Tensor dk_acc, at::Tensor dv_acc, double scale, at::Tensor kblk,
                  at::Tensor kpos, at::Tensor qoff) {
  c10::cuda::CUDAGuard guard(q.device());
  AttnBwdArgs a;
  a.f = attn_sel_args(q, k, v, o, lse, scale, kblk, kpos, qoff);
  const int64_t hd = q.size(3);
  attn_check(dout, "dout", hd);
  TORCH_CHECK(dout.sizes() == q.sizes(), "dout [E, Lq, nh, hd]");
  req(D, at::kFloat, "D");
  req(dq_acc, at::kFloat, "dq_acc");
  req(dk_acc, at::kFloat, "dk_acc");
  req(dv_acc, at::kFloat, "dv_acc");
  TORCH_CHECK(D.is_contiguous() && D.numel() == lse.numel(), "D [E, nh, Lq]");
  TORCH_CHECK(dq_acc.is_contiguous() && dq_acc.sizes() == q.sizes(), "dq_acc [E, Lq, nh, hd] fp32, contiguous");
  TORCH_CHECK(dk_acc.is_contiguous() && dk_acc.sizes() == k.sizes() && dv_acc.is_contiguous() &&
                  dv_acc.sizes() == v.sizes(),
              "dk_acc / dv_acc [B, Lsrc, nh, hd] fp32, contiguous");
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.sd_b = dout.stride(0); a.sd_l = dout.stride(1); a.sd_h = dout.stride(2);
  a.D = D.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dk = a.dv = nullptr;
  a.sdk_b = a.sdk_l = a.sdk_h = a.sdv_b = a.sdv_l = a.sdv_h = 0;
  a.dk_acc = dk_acc.data_ptr<float>();
  a.dv_acc = dv_acc.data_ptr<float>();
  a.kb_lsrc = (int)k.size(1);
  a.scale = (float)scale;
  const int rc = attn_bwd_launch(a, (int)hd, stream());
  TORCH_CHECK(rc == 0, "attn_sel_bwd launch failed (", rc, ")");
}

void attn_probsum(at::Tensor q, at::Tensor k, at::Tensor lse, at::Tensor imp, double scale, int64_t window,
                  int64_t q_offset, c10::optional<at::Tensor> kpos, c10::optional<at::Tensor> qoff) {
  c10::cuda::CUDAGuard guard(q.device());
  const AttnArgs a = attn_args(q, k, k, q, lse, scale, window, q_offset, kpos, qoff);
  req(imp, at::kFloat, "imp");
  TORCH_CHECK(imp.is_contiguous() && imp.dim() == 3 && imp.size(0) == q.size(0) && imp.size(1) == q.size(1) &&
                  imp.size(2) == k.size(1),
              "imp [B, Lq, Lk] fp32");
  const int rc = attn_probsum_launch(a, imp.data_ptr<float>(), (int)q.size(3), stream());
  TORCH_CHECK(rc == 0, "attn_probsum launch failed (", rc, ")");
}

// ---- gated delta rule chunk scan -----------------------------------------------------------
static void gdn_req(const at::Tensor& t, at::ScalarType dt, const char* name, std::initializer_list<int64_t> shape) {
  req(t, dt, name);
  TORCH_CHECK(t.is_contiguous() && t.sizes() == at::IntArrayRef(shape), name, " must be contiguous with shape ",
              at::IntArrayRef(shape), ", got ", t.sizes());
}

static GdnArgs gdn_args(const at::Tensor& qe, const at::Tensor& kc, const at::Tensor& kd, const at::Tensor& intra,
                        const at::Tensor& tot, int64_t HVD) {
  TORCH_CHECK(qe.dim() == 5 && qe.size(3) == 64, "qe [B, nh, nc, 64, HD]");
  const int64_t B = qe.size(0), nh = qe.size(1), nc = qe.size(2), HD = qe.size(4);
  TORCH_CHECK(HD == 64 || HD == 128, "key head dim must be 64 or 128");
  TORCH_CHECK(HVD % 64 == 0, "value head dim must be a multiple of 64");
  gdn_req(qe, at::kBFloat16, "qe", {B, nh, nc, 64, HD});
  gdn_req(kc, at::kBFloat16, "kc", {B, nh, nc, 64, HD});
  gdn_req(kd, at::kBFloat16, "kd", {B, nh, nc, 64, HD});
  gdn_req(intra, at::kBFloat16, "intra", {B, nh, nc, 64, 64});
  gdn_req(tot, at::kFloat, "tot", {B, nh, nc, HD});
  GdnArgs a{};
  a.qe = reinterpret_cast<const __nv_bfloat16*>(qe.data_ptr());
  a.kc = reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr());
  a.kd = reinterpret_cast<const __nv_bfloat16*>(kd.data_ptr());
  a.intra = reinterpret_cast<const __nv_bfloat16*>(intra.data_ptr());
  a.tot = tot.data_ptr<float>();
  a.B = (int)B; a.nh = (int)nh; a.nc = (int)nc; a.HVD = (int)HVD;
  return a;
}

void gdn_scan_fwd(at::Tensor qe, at::Tensor kc, at::Tensor kd, at::Tensor intra, at::Tensor vc, at::Tensor tot,
                  c10::optional<at::Tensor> S0, at::Tensor o, at::Tensor S_all, at::Tensor vnew, at::Tensor S_fin) {
  c10::cuda::CUDAGuard guard(qe.device());
  const int64_t HVD = vc.size(-1);
  GdnArgs a = gdn_args(qe, kc, kd, intra, tot, HVD);
  const int64_t B = a.B, nh = a.nh, nc = a.nc, HD = qe.size(4);
  gdn_req(vc, at::kFloat, "vc", {B, nh, nc, 64, HVD});
  gdn_req(o, at::kFloat, "o", {B, nh, nc, 64, HVD});
  gdn_req(vnew, at::kFloat, "vnew", {B, nh, nc, 64, HVD});
  gdn_req(S_all, at::kFloat, "S_all", {B, nh, nc, HVD, HD});
  gdn_req(S_fin, at::kFloat, "S_fin", {B, nh, HVD, HD});
  a.vc = vc.data_ptr<float>();
  a.S0 = nullptr;
  if (S0 && S0->defined()) {
    gdn_req(*S0, at::kFloat, "S0", {B, nh, HVD, HD});
    a.S0 = S0->data_ptr<float>();
  }
  a.o = o.data_ptr<float>(); a.S_all = S_all.data_ptr<float>(); a.vnew = vnew.data_ptr<float>();
  a.S_fin = S_fin.data_ptr<float>();
  const int rc = gdn_scan_launch(a, (int)HD, false, num_sms(qe), stream());
  TORCH_CHECK(rc == 0, "gdn_scan_fwd launch failed (", rc, ")");
}

void gdn_scan_bwd(at::Tensor qe, at::Tensor kc, at::Tensor kd, at::Tensor intra, at::Tensor tot, at::Tensor S_all,
                  at::Tensor vnew, at::Tensor dout, c10::optional<at::Tensor> dS_fin, at::Tensor dqe_p, at::Tensor dkc_p,
                  at::Tensor dkd_p, at::Tensor din_p, at::Tensor dtot_p, at::Tensor dvc, at::Tensor dS0) {
  c10::cuda::CUDAGuard guard(qe.device());
  const int64_t HVD = vnew.size(-1);
  GdnArgs a = gdn_args(qe, kc, kd, intra, tot, HVD);
  const int64_t B = a.B, nh = a.nh, nc = a.nc, HD = qe.size(4), nvb = HVD / gdn_scan_bwd_value_block();
  gdn_req(S_all, at::kFloat, "S_all", {B, nh, nc, HVD, HD});
  gdn_req(vnew, at::kFloat, "vnew", {B, nh, nc, 64, HVD});
  gdn_req(dout, at::kFloat, "dout", {B, nh, nc, 64, HVD});
  gdn_req(dqe_p, at::kFloat, "dqe_p", {nvb, B, nh, nc, 64, HD});
  gdn_req(dkc_p, at::kFloat, "dkc_p", {nvb, B, nh, nc, 64, HD});
  gdn_req(dkd_p, at::kFloat, "dkd_p", {nvb, B, nh, nc, 64, HD});
  gdn_req(din_p, at::kFloat, "din_p", {nvb, B, nh, nc, 64, 64});
  gdn_req(dtot_p, at::kFloat, "dtot_p", {nvb, B, nh, nc, HD});
  gdn_req(dvc, at::kFloat, "dvc", {B, nh, nc, 64, HVD});
  gdn_req(dS0, at::kFloat, "dS0", {B, nh, HVD, HD});
  a.S_all = S_all.data_ptr<float>(); a.vnew = vnew.data_ptr<float>(); a.dout = dout.data_ptr<float>();
  a.dS_fin = nullptr;
  if (dS_fin && dS_fin->defined()) {
    gdn_req(*dS_fin, at::kFloat, "dS_fin", {B, nh, HVD, HD});
    a.dS_fin = dS_fin->data_ptr<float>();
  }
  a.dqe_p = dqe_p.data_ptr<float>(); a.dkc_p = dkc_p.data_ptr<float>(); a.dkd_p = dkd_p.data_ptr<float>();
  a.din_p = din_p.data_ptr<float>(); a.dtot_p = dtot_p.data_ptr<float>(); a.dvc = dvc.data_ptr<float>();
  a.dS0 = dS0.data_ptr<float>();
  const int rc = gdn_scan_launch(a, (int)HD, true, num_sms(qe), stream());
  TORCH_CHECK(rc == 0, "gdn_scan_bwd launch failed (", rc, ")");
}

// ---- gated delta rule decode step ------------------------------------------------------------
void gdn_decode(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor beta, at::Tensor alog, at::Tensor S,
                at::Tensor o) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.dim() == 4 && v.dim() == 4, "q [B, T, nh, hd], v [B, T, nh, hvd]");
  const int64_t B = q.size(0), T = q.size(1), nh = q.size(2), hd = q.size(3), hvd = v.size(3);
  TORCH_CHECK(hd == 64 || hd == 128, "key head dim must be 64 or 128");
  const int64_t ad = alog.size(-1);
  TORCH_CHECK(ad == 1 || ad == hd, "alog: one decay per head or per key dim");
  gdn_req(q, at::kFloat, "q", {B, T, nh, hd});
  gdn_req(k, at::kFloat, "k", {B, T, nh, hd});
  gdn_req(v, at::kFloat, "v", {B, T, nh, hvd});
  gdn_req(beta, at::kFloat, "beta", {B, T, nh});
  gdn_req(alog, at::kFloat, "alog", {B, T, nh, ad});
  gdn_req(S, at::kFloat, "S", {B, nh, hvd, hd});
  gdn_req(o, at::kFloat, "o", {B, T, nh, hvd});
  GdnDecodeArgs a{q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), beta.data_ptr<float>(),
                  alog.data_ptr<float>(), S.data_ptr<float>(), o.data_ptr<float>(),
                  (int)B, (int)T, (int)nh, (int)hvd, (int)ad};
  const int rc = gdn_decode_launch(a, (int)hd, stream());
  TORCH_CHECK(rc == 0, "gdn_decode launch failed (", rc, ")");
}

// ---- per-key-dim-decay intra-chunk matrices -------------------------------------------------
static KdaArgs kda_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& kb, const at::Tensor& G) {
  TORCH_CHECK(q.dim() == 3 && q.size(1) == 64 && q.size(2) % 32 == 0, "q [N, 64, HD] with HD a multiple of 32");
  const int64_t N = q.size(0), HD = q.size(2);
  gdn_req(q, at::kFloat, "q", {N, 64, HD});
  gdn_req(k, at::kFloat, "k", {N, 64, HD});
  gdn_req(kb, at::kFloat, "kb", {N, 64, HD});
  gdn_req(G, at::kFloat, "G", {N, 64, HD});
  KdaArgs a{};
  a.q = q.data_ptr<float>(); a.k = k.data_ptr<float>(); a.kb = kb.data_ptr<float>(); a.G = G.data_ptr<float>();
  a.N = N; a.HD = (int)HD;
  return a;
}

void kda_intra_fwd(at::Tensor q, at::Tensor k, at::Tensor kb, at::Tensor G, at::Tensor intra, at::Tensor Lm) {
  c10::cuda::CUDAGuard guard(q.device());
  KdaArgs a = kda_args(q, k, kb, G);
  gdn_req(intra, at::kFloat, "intra", {a.N, 64, 64});
  gdn_req(Lm, at::kFloat, "Lm", {a.N, 64, 64});
  a.intra = intra.data_ptr<float>(); a.Lm = Lm.data_ptr<float>();
  const int rc = kda_intra_launch(a, false, stream());
  TORCH_CHECK(rc == 0, "kda_intra_fwd launch failed (", rc, ")");
}

void kda_intra_bwd(at::Tensor q, at::Tensor k, at::Tensor kb, at::Tensor G, at::Tensor gI, at::Tensor gL,
                   at::Tensor dq, at::Tensor dk, at::Tensor dkb, at::Tensor dG) {
  c10::cuda::CUDAGuard guard(q.device());
  KdaArgs a = kda_args(q, k, kb, G);
  const int64_t N = a.N, HD = a.HD;
  gdn_req(gI, at::kFloat, "gI", {N, 64, 64});
  gdn_req(gL, at::kFloat, "gL", {N, 64, 64});
  for (auto* t : {&dq, &dk, &dkb, &dG}) gdn_req(*t, at::kFloat, "gradient", {N, 64, HD});
  a.gI = gI.data_ptr<float>(); a.gL = gL.data_ptr<float>();
  a.dq = dq.data_ptr<float>(); a.dk = dk.data_ptr<float>(); a.dkb = dkb.data_ptr<float>(); a.dG = dG.data_ptr<float>();
  const int rc = kda_intra_launch(a, true, stream());
  TORCH_CHECK(rc == 0, "kda_intra_bwd launch failed (", rc, ")");
}

// ---- S5 complex diagonal scan ----------------------------------------------------------------
static const float2* c2(const at::Tensor& t) { return reinterpret_cast<const float2*>(t.data_ptr()); }
static float2* c2m(at::Tensor& t) { return reinterpret_cast<float2*>(t.data_ptr()); }

static S5Args s5_args(const at::Tensor& lam, int64_t B, int64_t L, int64_t P) {
  gdn_req(lam, at::kComplexFloat, "lam", {P});
  S5Args a{};
  a.lam = c2(lam);
  a.B = B; a.L = (int)L; a.P = (int)P; a.nchunk = (int)((L + 63) / 64);
  return a;
}

void s5_scan_fwd(at::Tensor lam, at::Tensor bu, c10::optional<at::Tensor> x0, at::Tensor xs, at::Tensor xlast,
                 at::Tensor part) {
  c10::cuda::CUDAGuard guard(bu.device());
  TORCH_CHECK(bu.dim() == 3, "bu [B, L, P]");
  const int64_t B = bu.size(0), L = bu.size(1), P = bu.size(2);
  S5Args a = s5_args(lam, B, L, P);
  gdn_req(bu, at::kComplexFloat, "bu", {B, L, P});
  gdn_req(xs, at::kComplexFloat, "xs", {B, L, P});
  gdn_req(xlast, at::kComplexFloat, "xlast", {B, P});
  gdn_req(part, at::kComplexFloat, "part", {B, a.nchunk, P});
  a.bu = c2(bu); a.xs = c2m(xs); a.xlast = c2m(xlast); a.part = c2m(part);
  a.x0 = nullptr;
  if (x0 && x0->defined()) {
    gdn_req(*x0, at::kComplexFloat, "x0", {B, P});
    a.x0 = c2(*x0);
  }
  const int rc = s5_scan_launch(a, false, stream());
  TORCH_CHECK(rc == 0, "s5_scan_fwd launch failed (", rc, ")");
}

void s5_scan_bwd(at::Tensor lam, at::Tensor xs, c10::optional<at::Tensor> x0, at::Tensor dxs,
                 c10::optional<at::Tensor> dxlast, at::Tensor dbu, at::Tensor dlam, c10::optional<at::Tensor> dx0,
                 at::Tensor part) {
  c10::cuda::CUDAGuard guard(xs.device());
  TORCH_CHECK(xs.dim() == 3, "xs [B, L, P]");
  const int64_t B = xs.size(0), L = xs.size(1), P = xs.size(2);
  S5Args a = s5_args(lam, B, L, P);
  gdn_req(xs, at::kComplexFloat, "xs", {B, L, P});
  gdn_req(dxs, at::kComplexFloat, "dxs", {B, L, P});
  gdn_req(dbu, at::kComplexFloat, "dbu", {B, L, P});
  gdn_req(dlam, at::kComplexFloat, "dlam", {P});
  gdn_req(part, at::kComplexFloat, "part", {B, a.nchunk, P});
  a.xs = c2m(xs); a.dxs = c2(dxs); a.dbu = c2m(dbu); a.dlam = c2m(dlam); a.part = c2m(part);
  a.x0 = nullptr; a.dxlast = nullptr; a.dx0 = nullptr;
  if (x0 && x0->defined()) { gdn_req(*x0, at::kComplexFloat, "x0", {B, P}); a.x0 = c2(*x0); }
  if (dxlast && dxlast->defined()) { gdn_req(*dxlast, at::kComplexFloat, "dxlast", {B, P}); a.dxlast = c2(*dxlast); }
  if (dx0 && dx0->defined()) { gdn_req(*dx0, at::kComplexFloat, "dx0", {B, P}); a.dx0 = c2m(*dx0); }
  const int rc = s5_scan_launch(a, true, stream());
  TORCH_CHECK(rc == 0, "s5_scan_bwd launch failed (", rc, ")");
}

// ---- profiling ---------------------------------------------------------------------------

// ---- decode / engine ----------------------------------------------------------------------
void m3_decode_step(at::Tensor proj, int64_t nh, at::Tensor wB, at::Tensor wC, at::Tensor dt_bias, at::Tensor Bb,
                    at::Tensor Cb, at::Tensor D, double A_floor, double eps, at::Tensor ang, at::Tensor ssm,
                    at::Tensor kprev, at::Tensor vprev, at::Tensor y, int64_t T) {
  req(proj, at::kBFloat16, "proj");
  req(ssm, at::kFloat, "ssm");
  req(y, at::kBFloat16, "y");
  c10::cuda::CUDAGuard guard(proj.device());
  int64_t B = proj.size(0);
  TORCH_CHECK(ssm.numel() * T == B * nh * M3_P * M3_N, "state shape");
  B /= T;
  if (T > 1) {
    TORCH_CHECK(T <= 8, "at most 8 tokens per multi-token decode step");
    m3_decode_multi_launch(proj.data_ptr(), (int)B, (int)T, (int)proj.size(1), (int)nh, wB.data_ptr<float>(),
                           wC.data_ptr<float>(), dt_bias.data_ptr<float>(), Bb.data_ptr<float>(),
                           Cb.data_ptr<float>(), D.data_ptr<float>(), (float)A_floor, (float)eps,
                           ang.data_ptr<float>(), ssm.data_ptr<float>(), kprev.data_ptr<float>(),
                           vprev.data_ptr<float>(), y.data_ptr(), stream());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  m3_decode_step_launch(proj.data_ptr(), (int)B, (int)proj.size(1), (int)nh, wB.data_ptr<float>(),
                        wC.data_ptr<float>(), dt_bias.data_ptr<float>(), Bb.data_ptr<float>(), Cb.data_ptr<float>(),
                        D.data_ptr<float>(), (float)A_floor, (float)eps, ang.data_ptr<float>(), ssm.data_ptr<float>(),
                        kprev.data_ptr<float>(), vprev.data_ptr<float>(), y.data_ptr(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void eng_process(at::Tensor asks, at::Tensor bids, at::Tensor trades, at::Tensor msgs, int64_t init_id,
                 int64_t book_depth, int64_t cancel_mode, int64_t type4, bool check_fill) {
  req(asks, at::kInt, "asks");
  req(bids, at::kInt, "bids");
  req(trades, at::kInt, "trades");
  req(msgs, at::kInt, "msgs");
  TORCH_CHECK(asks.size(1) <= 128 && trades.size(1) <= 128, "at most 128 rows per side / trades");
  TORCH_CHECK(cancel_mode <= 1, "cancel modes 2/3 (random fallback) run on the CPU engine");
  c10::cuda::CUDAGuard guard(asks.device());
  int64_t nb = asks.size(0);
  eng_process_launch(asks.data_ptr<int>(), bids.data_ptr<int>(), trades.data_ptr<int>(), msgs.data_ptr<int>(),
                     (int)msgs.size(1), (int)nb, (int)asks.size(1), (int)trades.size(1), (int)init_id,
                     (int)book_depth, (int)cancel_mode, (int)type4, check_fill ? 1 : 0, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor eng_l2(at::Tensor asks, at::Tensor bids, int64_t levels) {
  req(asks, at::kInt, "asks");
  c10::cuda::CUDAGuard guard(asks.device());
  auto out = at::empty({asks.size(0), 4 * levels}, asks.options());
  eng_l2_launch(asks.data_ptr<int>(), bids.data_ptr<int>(), out.data_ptr<int>(), (int)levels, (int)asks.size(0),
                (int)asks.size(1), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void gen_apply(at::Tensor asks, at::Tensor bids, at::Tensor trades, at::Tensor toks, std::vector<int64_t> lay,
               int64_t init_id, int64_t book_depth, int64_t cancel_mode, int64_t type4, bool check_fill,
               at::Tensor new_oid, at::Tensor p_mid, at::Tensor time_in, at::Tensor raw_out, at::Tensor msg_out,
               at::Tensor prov_out, at::Tensor l2_out, at::Tensor img_out, bool apply,
               c10::optional<at::Tensor> inject) {
  req(asks, at::kInt, "asks");
  req(bids, at::kInt, "bids");
  req(trades, at::kInt, "trades");
  req(toks, at::kLong, "toks");
  req(p_mid, at::kInt, "p_mid");
  req(time_in, at::kInt, "time_in");
  req(raw_out, at::kInt, "raw_out");
  req(msg_out, at::kInt, "msg_out");
  req(prov_out, at::kInt, "prov_out");
  req(l2_out, at::kInt, "l2_out");
  req(new_oid, at::kInt, "new_oid");
  TORCH_CHECK(img_out.is_cuda() && img_out.scalar_type() == at::kFloat && img_out.stride(1) == 1, "img_out");
  TORCH_CHECK(lay.size() == 22, "layout has 22 entries");
  TORCH_CHECK(asks.size(1) <= 128 && trades.size(1) <= 128, "at most 128 rows per side / trades");
  TORCH_CHECK(cancel_mode <= 1, "cancel modes 2/3 run on the CPU engine");
  GenLayout L;
  int* f = &L.msg_len;
  for (int i = 0; i < 22; ++i) f[i] = (int)lay[i];
  TORCH_CHECK(L.msg_len <= 32 && L.l2_levels <= 64 && L.price_digits <= 4, "layout out of range");
  TORCH_CHECK(toks.size(1) == L.msg_len, "toks width");
  TORCH_CHECK(img_out.size(1) >= 3 + L.img_levels, "img_out width");
  TORCH_CHECK(l2_out.size(1) == 4 * L.l2_levels, "l2_out width");
  const int* injp = nullptr;
  if (inject.has_value() && inject->defined()) {
    req(*inject, at::kInt, "inject");
    TORCH_CHECK(inject->numel() == 5, "inject = [flag, event_type, side, qty, offset_ticks]");
    injp = inject->data_ptr<int>();
  }
  c10::cuda::CUDAGuard guard(asks.device());
  gen_apply_launch(asks.data_ptr<int>(), bids.data_ptr<int>(), trades.data_ptr<int>(), toks.data_ptr<int64_t>(), L,
                   (int)asks.size(1), (int)trades.size(1), (int)init_id, (int)book_depth, (int)cancel_mode,
                   (int)type4, check_fill ? 1 : 0, new_oid.data_ptr<int>(), p_mid.data_ptr<int>(),
                   time_in.data_ptr<int>(), raw_out.data_ptr<int>(), msg_out.data_ptr<int>(),
                   prov_out.data_ptr<int>(), l2_out.data_ptr<int>(), img_out.data_ptr<float>(),
                   (int)img_out.stride(0), (int)asks.size(0), apply ? 1 : 0, injp, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gen_sample(at::Tensor logits, c10::optional<at::Tensor> bias, at::Tensor allow, int64_t seed, at::Tensor ctr,
                int64_t salt, int64_t top_n, at::Tensor out, int64_t out_offset, int64_t out_stride) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "logits");
  req(allow, at::kByte, "allow");
  req(ctr, at::kLong, "ctr");
  req(out, at::kLong, "out");
  TORCH_CHECK(top_n == 1 || top_n == -1, "device sampler supports top_n 1 (argmax) and -1 (full)");
  int64_t V = logits.size(1);
  TORCH_CHECK(allow.numel() == V, "mask width");
  TORCH_CHECK(out_offset + (logits.size(0) - 1) * out_stride < out.numel(), "out too small");
  const float* bp = nullptr;
  if (bias.has_value()) {
    req(*bias, at::kFloat, "bias");
    TORCH_CHECK(bias->numel() == V, "bias width");
    bp = bias->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(logits.device());
  gen_sample_launch(logits.data_ptr<float>(), (int)logits.stride(0), bp, allow.data_ptr<unsigned char>(), (int)V,
                    (int)logits.size(0), (unsigned long long)seed, reinterpret_cast<const long long*>(ctr.data_ptr<int64_t>()), (int)salt, (int)top_n,
                    out.data_ptr<int64_t>() + out_offset, (int)out_stride, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gen_time_tokens(at::Tensor msg, int64_t dt_pos, int64_t time_off, at::Tensor time) {
  req(msg, at::kLong, "msg");
  req(time, at::kInt, "time");
  c10::cuda::CUDAGuard guard(msg.device());
  gen_time_tokens_launch(msg.data_ptr<int64_t>(), (int)msg.size(1), (int)dt_pos, (int)time_off,
                         time.data_ptr<int>(), (int)msg.size(0), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_fused_adam(std::vector<int64_t> G, std::vector<int64_t> P, std::vector<int64_t> S,
                   std::vector<int64_t> flags, std::vector<int64_t> sums, at::Tensor m, at::Tensor v,
                   at::Tensor scratch, at::Tensor status, int64_t lo, int64_t hi, int64_t n_ssm, int64_t rank,
                   int64_t seq, int64_t spin_limit, double lr_s, double lr_r, double wd, double b1, double b2,
                   double eps, double bc1, double bc2, double max_norm) {
  const int world = (int)G.size();
  TORCH_CHECK(world >= 1 && world <= DPF_MAXW, "world size must be in [1, ", DPF_MAXW, "]");
  TORCH_CHECK((int)P.size() == world && (int)S.size() == world && (int)flags.size() == world &&
                  (int)sums.size() == world, "one pointer per rank for every buffer");
  req(m, at::kFloat, "m");
  req(v, at::kFloat, "v");
  req(scratch, at::kInt, "scratch");
  req(status, at::kInt, "status");
  TORCH_CHECK(lo % 128 == 0 && hi % 4 == 0 && hi >= lo && m.numel() == hi - lo && v.numel() == hi - lo,
              "shard bounds / moment sizes");
  TORCH_CHECK(scratch.numel() >= 2, "scratch holds [sumsq, abort]");
  c10::cuda::CUDAGuard guard(m.device());
  DpfArgs a{};
  for (int k = 0; k < world; ++k) {
    a.G[k] = reinterpret_cast<float*>(G[k]);
    a.P[k] = reinterpret_cast<float*>(P[k]);
    a.S[k] = reinterpret_cast<__nv_bfloat16*>(S[k]);
    a.flags[k] = reinterpret_cast<int*>(flags[k]);
    a.sums[k] = reinterpret_cast<float*>(sums[k]);
    TORCH_CHECK(G[k] % 16 == 0 && P[k] % 16 == 0 && S[k] % 8 == 0, "buffers must be 16-byte aligned");
  }
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.sumsq_local = reinterpret_cast<float*>(scratch.data_ptr<int>());
  a.abort = scratch.data_ptr<int>() + 1;
  a.status = status.data_ptr<int>();
  a.lo = lo; a.hi = hi; a.n_ssm = n_ssm;
  a.world = world; a.rank = (int)rank; a.seq = (int)seq; a.spin_limit = spin_limit;
  a.lr_s = (float)lr_s; a.lr_r = (float)lr_r; a.wd = (float)wd; a.b1 = (float)b1; a.b2 = (float)b2;
  a.eps = (float)eps; a.bc1 = (float)bc1; a.bc2 = (float)bc2; a.max_norm = (float)max_norm;
  a.inv_world = 1.f / world;
  C10_CUDA_CHECK(cudaMemsetAsync(scratch.data_ptr<int>(), 0, 2 * sizeof(int), stream()));
  int rc = dp_fused_adam_launch(a, num_sms(m), stream());
  TORCH_CHECK(rc == 0, "dp_fused_adam launch failed: ", rc > 0 ? cudaGetErrorString((cudaError_t)rc) : "occupancy");
}

// ---- embedding gathers -------------------------------------------------------------------
at::Tensor embed_sum_fwd(std::vector<at::Tensor> tables, at::Tensor idx) {
  TORCH_CHECK(!tables.empty() && (int)tables.size() <= EMBED_MAX_FIELDS, "1..", EMBED_MAX_FIELDS, " tables");
  req(idx, at::kLong, "idx");
  c10::cuda::CUDAGuard guard(idx.device());
  const int nf = (int)tables.size();
  const int64_t D = tables[0].size(1);
  TORCH_CHECK(idx.size(-1) == nf, "idx [..., n_fields]");
  EmbedSumArgs a{};
  for (int f = 0; f < nf; ++f) {
    req(tables[f], at::kFloat, "table");
    TORCH_CHECK(tables[f].dim() == 2 && tables[f].size(1) == D, "tables [rows, D] with one D");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(tables[f].data_ptr()) % 16 == 0, "tables must be 16-byte aligned");
    a.tab[f] = tables[f].data_ptr<float>();
    a.rows[f] = (int)tables[f].size(0);
  }
  const int64_t T = idx.numel() / nf;
  auto sizes = idx.sizes().vec();
  sizes.back() = D;
  auto out = at::empty(sizes, tables[0].options());
  a.nf = nf; a.D = (int)D; a.idx = reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()); a.out = out.data_ptr<float>(); a.T = T;
  const int rc = embed_sum_fwd_launch(a, stream());
  TORCH_CHECK(rc == 0, "embed_sum_fwd failed (", rc, "): D must be a multiple of 4");
  return out;
}

void embed_sum_bwd(std::vector<at::Tensor> grads, at::Tensor dout, at::Tensor idx) {
  req(idx, at::kLong, "idx");
  req(dout, at::kFloat, "dout");
  c10::cuda::CUDAGuard guard(idx.device());
  const int nf = (int)grads.size();
  TORCH_CHECK(nf >= 1 && nf <= EMBED_MAX_FIELDS && idx.size(-1) == nf, "one gradient table per field");
  const int64_t D = dout.size(-1);
  EmbedSumBwdArgs a{};
  for (int f = 0; f < nf; ++f) {
    req(grads[f], at::kFloat, "grad");
    TORCH_CHECK(grads[f].dim() == 2 && grads[f].size(1) == D, "gradient tables [rows, D]");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(grads[f].data_ptr()) % 16 == 0, "gradients must be 16-byte aligned");
    a.gtab[f] = grads[f].data_ptr<float>();
    a.rows[f] = (int)grads[f].size(0);
  }
  a.nf = nf; a.D = (int)D; a.idx = reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()); a.dout = dout.data_ptr<float>();
  a.T = idx.numel() / nf;
  const int rc = embed_sum_bwd_launch(a, stream());
  TORCH_CHECK(rc == 0, "embed_sum_bwd failed (", rc, ")");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sigma0_b200 sm_100a kernels";
  m.def("m3_fwd", &m3_fwd, py::arg("proj"), py::arg("B"), py::arg("L"), py::arg("nh"), py::arg("wB"), py::arg("wC"),
        py::arg("dt_bias"), py::arg("Bb"), py::arg("Cb"), py::arg("D"), py::arg("A_floor"), py::arg("eps"),
        py::arg("want_final") = false, py::arg("return_prep") = false, py::arg("init_state") = py::none(),
        py::arg("init_angle") = py::none(),
        "Mamba3 SSD forward -> (y, states, final state, final angle[, prep...]); init_state [B, nh, P, N] and "
        "init_angle [B, nh, R] continue a sequence from a carry");
  m.def("m3_bwd", &m3_bwd, py::arg("proj"), py::arg("dy"), py::arg("wB"), py::arg("wC"), py::arg("dt_bias"),
        py::arg("Bb"), py::arg("Cb"), py::arg("D"), py::arg("B"), py::arg("L"), py::arg("nh"), py::arg("A_floor"),
        py::arg("eps"), py::arg("saved_states") = py::none(), py::arg("saved_prep") = py::none(),
        py::arg("d_final") = py::none(), py::arg("want_d_init") = false, py::arg("final_state") = py::none(),
        "Mamba3 SSD backward -> (dproj, dB_norm, dC_norm, ddt_bias, dD, dC_bias, dB_bias[, d_init_state, "
        "d_init_angle]); d_final: gradient of the final state");
  m.def("embed_sum_fwd", &embed_sum_fwd, "sum over fields of each field table's row: [..., nf] ids -> [..., D]");
  m.def("embed_sum_bwd", &embed_sum_bwd, "scatter-add of the output gradient into each field table's gradient");
  m.def("ln_fwd", &ln_fwd);
  m.def("ln_bwd", &ln_bwd);
  m.def("rms_fwd", &rms_fwd);
  m.def("rms_bwd", &rms_bwd);
  m.def("gelu_fwd", &gelu_fwd);
  m.def("glu_res_fwd", &glu_res_fwd);
  m.def("glu_res_bwd", &glu_res_bwd);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("ce_fwd_bwd", &ce_fwd_bwd);
  m.def("sumsq", &sumsq);
  m.def("adam", &adam);
  m.def("tp_gemm_allreduce", &tp_gemm_allreduce, py::arg("A"), py::arg("Bt"), py::arg("recv"), py::arg("rows_own"),
        py::arg("out"), py::arg("flags"), py::arg("rank"), py::arg("seq"), py::arg("spin_limit"), py::arg("status"),
        py::arg("abort"), py::arg("stamps") = py::none(),
        "out = sum over ranks of A_r Bt_r^T: tcgen05 tiles reduced into the owners' peer buffers, then all-gathered "
        "(cooperative launch; returns 0 or a launch error)");
  m.def("attn_fwd", &attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("scale"), py::arg("window"), py::arg("q_offset"), py::arg("kpos") = py::none(),
        py::arg("qoff") = py::none(),
        "causal / sliding-window flash attention forward: o and the base-2 row log-sum-exp (window <= 0: none; "
        "optional per-key positions and per-entry query offsets)");
  m.def("attn_bwd", &attn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("dout"), py::arg("D"), py::arg("dq_acc"), py::arg("dk"), py::arg("dv"), py::arg("scale"),
        py::arg("window"), py::arg("q_offset"), py::arg("kpos") = py::none(), py::arg("qoff") = py::none(),
        "flash attention backward: dk, dv written, dq accumulated into the zeroed fp32 dq_acc (scaled)");
  m.def("attn_sel_fwd", &attn_sel_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("scale"), py::arg("kblk"), py::arg("kpos"), py::arg("qoff"),
        "flash attention forward over block-indirect keys: entry e reads the 64-key blocks kblk[e] of source "
        "batch e / (E / B) (the NSA selected branch without a gather)");
  m.def("attn_sel_bwd", &attn_sel_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("dout"), py::arg("D"), py::arg("dq_acc"), py::arg("dk_acc"), py::arg("dv_acc"), py::arg("scale"),
        py::arg("kblk"), py::arg("kpos"), py::arg("qoff"),
        "its backward: dq into the zeroed fp32 dq_acc, dk / dv added into the zeroed fp32 source-shaped buffers");
  m.def("attn_probsum", &attn_probsum, py::arg("q"), py::arg("k"), py::arg("lse"), py::arg("imp"), py::arg("scale"),
        py::arg("window"), py::arg("q_offset"), py::arg("kpos") = py::none(), py::arg("qoff") = py::none(),
        "head-summed softmax probabilities [B, Lq, Lk] of a finished forward (no gradient)");
  m.def("gdn_scan_fwd", &gdn_scan_fwd,
        "gated delta rule cross-chunk scan: o, the chunk-start states, vnew and the final state");
  m.def("gdn_scan_bwd_value_block", &gdn_scan_bwd_value_block,
        "value rows per CTA of the reverse scan (the leading dimension of its partials is HVD / this)");
  m.def("gdn_scan_bwd", &gdn_scan_bwd,
        "reverse scan: per value-block partial gradients of qe / kc / kd / intra / tot, dvc and dS0");
  m.def("gdn_decode", &gdn_decode, "gated delta rule recurrent step over T tokens (state updated in place)");
  m.def("kda_intra_fwd", &kda_intra_fwd, "per-key-dim-decay intra-chunk score and WY matrices of 64-step chunks");
  m.def("kda_intra_bwd", &kda_intra_bwd, "gradients of q, k, kb and the cumulative log decay G");
  m.def("s5_scan_fwd", &s5_scan_fwd, "S5 complex diagonal recurrence: all states and the final one");
  m.def("s5_scan_bwd", &s5_scan_bwd, "reverse recurrence: dBu, dlam (accumulated into the zeroed dlam), dx0");
  m.def("m3_decode_step", &m3_decode_step, py::arg("proj"), py::arg("nh"), py::arg("wB"), py::arg("wC"),
        py::arg("dt_bias"), py::arg("Bb"), py::arg("Cb"), py::arg("D"), py::arg("A_floor"), py::arg("eps"),
        py::arg("ang"), py::arg("ssm"), py::arg("kprev"), py::arg("vprev"), py::arg("y"), py::arg("T") = 1,
        "Mamba3 recurrent step over T tokens (proj rows [B*T, ldp]; states updated in place)");
  m.def("eng_process", &eng_process, "batched matching engine: apply [B, M, 8] messages, one warp per book");
  m.def("eng_l2", &eng_l2, "batched L2 extraction");
  m.def("m3_use_tc", [](c10::optional<bool> on) { g_m3_tc = on.has_value() ? (*on ? 1 : 0) : -1; },
        py::arg("on") = py::none(),
        "Mamba3 SSD: True the tcgen05 chunk walkers, False the chunk-parallel kernels, None by occupancy");
  m.def("gemm_tc", &gemm_tc, "C (+)= A . B on the tcgen05 GEMM", py::arg("a"), py::arg("b"), py::arg("a_mn"),
        py::arg("b_mn"), py::arg("out_mode") = 0, py::arg("out") = c10::nullopt, py::arg("split_k") = 1);  // split_k 0: auto
  m.def("gemm_status", [](at::Tensor like) { return gemm_status(like); }, "status word of the tcgen05 GEMM");
  m.def("gemm_gelu_fwd", &gemm_gelu_fwd, "o = x . w and g = gelu(o) in one tcgen05 GEMM");
  m.def("gemm_ag", &gemm_ag, "y = x . W with W's row blocks all-gathered from the ranks inside the tcgen05 GEMM",
        py::arg("x"), py::arg("wfull"), py::arg("src"), py::arg("ready"), py::arg("counters"), py::arg("rank"),
        py::arg("seq"), py::arg("spin"));
  m.def("gemm_use_pair", [](bool on) { gemm_tc_set_pair(on ? 1 : 0); },
        "two-SM (cta_group::2) GEMM tiles (default) or one-SM tiles");
  m.def("m3_tc_status", [](at::Tensor like) { return m3_status(like); },
        "status word of the tcgen05 SSD kernels on the tensor's device (nonzero: a bounded wait gave up)");
  m.def("dp_fused_adam", &dp_fused_adam, "fused reduce-scatter + AdamW + all-gather over peer memory");
  m.def("gen_apply", &gen_apply, "generation: decode message tokens, match, L2 and next book image");
  m.def("gen_sample", &gen_sample, "syntax-masked argmax / Gumbel-max sampling from fp32 logits");
  m.def("gen_time_tokens", &gen_time_tokens, "generation: absolute-time tokens from delta-t tokens");
}
