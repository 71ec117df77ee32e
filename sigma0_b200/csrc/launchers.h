// Raw-pointer launch entry points of the sm_100a kernels.  The CUDA sources
// include no torch headers (fast, parallel compiles); tensor handling lives in
// bindings.cpp.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// ---- Mamba3 SSD (mamba3_ssd.cu) -------------------------------------------------------
struct M3Geo {
  int B, L, nh;
  int ldp;   // row stride (elements) of proj / dproj
};
struct M3Scan {
  const void* proj;
  const void* bc;
  const float *dt, *adt, *sig, *rate;
  const float *Bb, *Cb, *D;
  const float* theta0;   // [B, nh, nc, R]
  const float* aend;     // [B, nh, nc]
};
struct M3BwdOut {
  void* dproj;
  void *gQ, *gK;
  float *dthl, *dthtot;
  float *dgam, *dscl, *dadt;
  float *dD, *dCb, *dBb;
};
int m3_nchunks(int L);

// tcgen05 chunk walker (mamba3_tc.cu): the whole SSD forward / backward in one kernel each
struct M3TcFwd {
  const void* proj;                         // [B, L, ldp] bf16
  const void* bc;                           // [B, L, 2N] bf16 (BCNorm'd B | C)
  const float *dt, *adt, *sig;              // [B, nh, lds]
  const float* rate;                        // [B, L, R]
  const float *Bb, *Cb, *D;
  void* y;                                  // [B, L, nh * P] bf16
  void* states;                             // [B, nh, nc] swizzled bf16 S_in images (backward) or null
  float* theta0;                            // [B, nh, nc, R] or null
  const float* s0;                          // [B, nh, P, N] initial state or null
  const float* th_in;                       // [B, nh, R] initial angle or null
  float* fin;                               // [B, nh, P, N] final state or null
  float* thf;                               // [B, nh, R] final angle or null
  int* status;                              // set to 1 when a bounded wait gave up
  int B, L, nh, ldp, lds;
  int nseg = 1, seg_lo = 0, seg_hi = 0;     // segments per sequence; walk segments [lo, hi) (hi 0: all)
};
int m3_fwd_tc_launch(const M3TcFwd& f, cudaStream_t st);   // 0, -3 (alignment), -4 (tensor map), -5 (segments), CUDA error
struct M3TcBwd {
  const void *proj, *bc, *dy;               // dy: [B, L, nh * P] bf16
  const float *dt, *adt, *sig, *rate, *Bb, *Cb, *D;
  const void* states;                       // the forward's S_in images
  const float* theta0;                      // the forward's chunk-start angles [B, nh, nc, R]
  const float* ds_fin;                      // [B, nh, P, N] gradient of the final state or null
  const float* s_fin;                       // [B, nh, P, N] the final state (needed with ds_fin) or null
  float* ds0;                               // [B, nh, P, N] gradient of the initial state or null
  void* dproj;                              // [B, L, ldp] bf16: z and x columns written
  void *gQ, *gK;                            // [B, L, nh * N] bf16
  float *dthl, *dthtot, *dgam, *dscl, *dadt;
  float *dD, *dCb, *dBb;                    // [B, nh], [B, nh, N], [B, nh, N]
  int* status;
  int B, L, nh, ldp, lds;
  int nseg = 1, seg_lo = 0, seg_hi = 0;
};
int m3_bwd_tc_launch(const M3TcBwd& f, cudaStream_t st);
void m3_prep_fwd_launch(const M3Geo& g, const void* proj, const float* wB, const float* wC,
                        const float* dt_bias, float A_floor, float eps, void* bc, float* dt, float* adt,
                        float* sig, float* rate, cudaStream_t st);
void m3_chunk_totals_launch(const M3Geo& g, const M3Scan& s, float* aend, float* angtot, float* theta0,
                            cudaStream_t st);
void m3_states_launch(const M3Geo& g, const M3Scan& s, void* states, cudaStream_t st,
                      float* final_state = nullptr);
void m3_scan_launch(const M3Geo& g, const M3Scan& s, const void* states, void* y, cudaStream_t st);
void m3_dstates_launch(const M3Geo& g, const M3Scan& s, const void* dy, void* U, cudaStream_t st);
void m3_chunk_bwd_launch(const M3Geo& g, const M3Scan& s, const void* dy, const void* states, const void* dsout,
                         const M3BwdOut& o, cudaStream_t st);
void m3_rev_carry_launch(const M3Geo& g, float* dthtot, cudaStream_t st);   // exclusive reverse scan over chunks
void m3_prep_bwd_launch(const M3Geo& g, const void* proj, const float* wB, const float* wC,
                        const float* dt_bias, float A_floor, float eps, const void* gQ, const void* gK,
                        const float* dthl, const float* dthc, const float* dgam, const float* dscl,
                        const float* dadt, void* dproj, float* dwB, float* dwC, float* ddt_bias,
                        cudaStream_t st);

// ---- embedding gathers (embed.cu) --------------------------------------------------------
#define EMBED_MAX_FIELDS 32
struct EmbedSumArgs {
  const float* tab[EMBED_MAX_FIELDS];   // one fp32 table [rows_f, D] per field
  int rows[EMBED_MAX_FIELDS];
  int nf, D;
  const long long* idx;                 // [T, nf] row ids
  float* out;                           // [T, D] = sum over fields of tab_f[idx[t, f]]
  long long T;
};
struct EmbedSumBwdArgs {
  float* gtab[EMBED_MAX_FIELDS];        // gradient of each table (accumulated)
  int rows[EMBED_MAX_FIELDS];
  int nf, D;
  const long long* idx;
  const float* dout;                    // [T, D]
  long long T;
};
int embed_sum_fwd_launch(const EmbedSumArgs& a, cudaStream_t st);
int embed_sum_bwd_launch(const EmbedSumBwdArgs& a, cudaStream_t st);

// ---- fused row/elementwise ops, loss and optimizer (fused_ops.cu) -------------------
void ln_fwd_launch(const float* x, const float* w, const float* b, void* y, float* mean, float* rstd, long T,
                   int D, float eps, int sms, cudaStream_t st);
int col_blocks(long T, int sms);   // blocks (= partial rows) of the column-reduction kernels
void ln_bwd_launch(const void* dy, const float* x, const float* mean, const float* rstd, const float* w,
                   const float* dres, float* dx, float* dw, float* db, float* part, long T, int D, int sms,
                   cudaStream_t st);
void rms_fwd_launch(const void* x, const float* w, void* y, float* rstd, long T, int D, float eps, int sms,
                    cudaStream_t st);
void rms_bwd_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                    float* part, long T, int D, int sms, cudaStream_t st);
void gelu_fwd_launch(const void* o, void* g, long n, int sms, cudaStream_t st);
void glu_res_fwd_launch(const float* x, const void* g, const void* h, const float* b, float* out, long n, int D,
                        int sms, cudaStream_t st);
int glu_bwd_blocks(long T, int sms);
void glu_res_bwd_launch(const float* dout, const void* g, const void* h, const float* b, void* dh, float* dgp,
                        float* db, float* part, long T, int D, int sms, cudaStream_t st);
void gelu_bwd_launch(const void* o, const float* dgp, const void* dgm, void* dout, long n, int sms,
                     cudaStream_t st);
void ce_launch(void* logits, const float* bias, const int64_t* labels, const float* wrow, float* loss, long T,
               int V, int ld, cudaStream_t st);
void sumsq_launch(const float* g, long n, float* out, int sms, cudaStream_t st);
void adam_launch(float* p, const float* g, float* m, float* v, void* pb, long n, const float* sumsq,
                 float max_norm, const float* lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                 int sms, cudaStream_t st);

// ---- Mamba3 decode step (decode.cu) ---------------------------------------------------
void m3_decode_step_launch(const void* proj, int B, int ldp, int nh, const float* wB, const float* wC,
                           const float* dt_bias, const float* Bb, const float* Cb, const float* D, float A_floor,
                           float eps, float* ang, float* ssm, float* kprev, float* vprev, void* y,
                           cudaStream_t st);

// ---- batched matching engine (engine.cu) ------------------------------------------------
void eng_process_launch(int* asks, int* bids, int* trades, const int* msgs, int n_msgs, int n_books, int n_orders,
                        int n_trades, int init_id, int book_depth, int cancel_mode, int type4, int check_fill,
                        cudaStream_t st);
void eng_l2_launch(const int* asks, const int* bids, int* out, int levels, int n_books, int n_orders,
                   cudaStream_t st);

// Token layout of one message for the generation step (positions and field
// token offsets of the active tokenizer mode).
struct GenLayout {
  int msg_len, fused_ed, ev_pos, ev_off, dir_pos, dir_off;
  int sign_off, price_off, price_digits, p_pos, pref_pos;
  int size_digits, size_off, size_n, s_pos, sref_pos;
  int time_off, dt_pos, tref_pos;
  int tick, img_levels, l2_levels;
};
void gen_apply_launch(int* asks, int* bids, int* trades, const int64_t* toks, const GenLayout& L, int n_orders,
                      int n_trades, int init_id, int book_depth, int cancel_mode, int type4, int check_fill,
                      const int* new_oid, int* p_mid, const int* time_in, int* raw_out, int* msg_out, int* prov_out,
                      int* l2_out, float* img_out, int img_stride, int n_books, int apply, const int* inj,
                      cudaStream_t st);

// generation (generate.cu)
void gen_sample_launch(const float* logits, int ldl, const float* bias, const unsigned char* allow, int V, int B,
                       unsigned long long seed, const long long* ctr, int salt, int top_n, int64_t* out,
                       int out_stride, cudaStream_t st);
void gen_time_tokens_launch(int64_t* msg, int msg_len, int dt_pos, int time_off, int* time, int n,
                            cudaStream_t st);

// fused data-parallel gradient sync + AdamW over peer memory (dp_fused.cu)
#define DPF_MAXW 8
struct DpfArgs {
  float* G[DPF_MAXW];          // every rank's flat gradient (peer-mapped)
  float* P[DPF_MAXW];          // every rank's flat fp32 parameters
  __nv_bfloat16* S[DPF_MAXW];  // every rank's bf16 shadow (or null)
  int* flags[DPF_MAXW];        // every rank's flag words [3][DPF_MAXW]
  float* sums[DPF_MAXW];       // every rank's sum-of-squares slots [DPF_MAXW]
  float* m;                    // this rank's Adam moments for [lo, hi)
  float* v;
  float* sumsq_local;          // zeroed before the launch
  int* abort;                  // zeroed before the launch
  int* status;                 // 0 = ok, 100 + phase = a peer did not arrive
  long lo, hi, n_ssm;
  int world, rank, seq;
  long long spin_limit;
  float lr_s, lr_r, wd, b1, b2, eps, bc1, bc2, max_norm, inv_world;
};
int dp_fused_adam_launch(const DpfArgs& a, int sms, cudaStream_t st);

void m3_decode_multi_launch(const void* proj, int B, int T, int ldp, int nh, const float* wB, const float* wC,
                            const float* dt_bias, const float* Bb, const float* Cb, const float* D, float A_floor,
                            float eps, float* ang, float* ssm, float* kprev, float* vprev, void* y,
                            cudaStream_t st);
int rms_wide_blocks(long T, int sms);
void rms_fwd_wide_launch(const void* x, const float* w, void* y, float* rstd, long T, int D, float eps, int sms,
                         cudaStream_t st);
void rms_bwd_wide_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                         float* part, long T, int D, int sms, cudaStream_t st);
void rms_bwd_pipe_launch(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw,
                         float* part, long T, int D, int sms, cudaStream_t st);
void ln_bwd_pipe_launch(const void* dy, const float* x, const float* mean, const float* rstd, const float* w,
                        const float* dres, float* dx, float* dw, float* db, float* part, long T, int D, int sms,
                        cudaStream_t st);

// dense bf16 GEMM on tcgen05 (gemm_tc.cu): C (+)= A . B with fp32 accumulation.
// A is [M, K] K-major (row-major, leading dimension lda) or, with a_mn, stored [K, M] MN-major;
// B is [N, K] K-major or, with b_mn, stored [K, N] MN-major.  C is written over its first
// c_rows x c_cols entries (c_rows <= M, c_cols <= N; leading dimension ldc): out_mode 0 bf16
// store, 1 fp32 store, 2 fp32 reduce-add (split_k > 1 only with 2), 3 bf16 store plus its GELU.  Bases 16-byte aligned,
// leading dimensions multiples of 16 bytes.
struct GemmArgs {
  const void* A;
  const void* B;
  void* C;
  int M, N, K;
  long lda, ldb, ldc;
  int c_rows, c_cols;
  int a_mn, b_mn;
  int out_mode;
  int split_k;
  int* status;                 // 1: a pipeline wait timed out
  // out_mode 3 (the GLU block's fused epilogue) also writes C2 = gelu(C) (bf16, leading
  // dimension ldc2)
  void* C2;
  long ldc2;
  // fused all-gather of B (ag_world > 1; two-SM kernel, B MN-major): B is this GPU's full
  // [K, N] buffer (leading dimension ldb == N), whose row block r (ag_rows rows) is copied in
  // by the kernel from ag_src[r] -- rank r's shard, a peer address for r != ag_rank -- once
  // ag_ready[r] (rank r's flag, a peer address) has reached ag_seq; ag_count (ag_world local
  // ints, zeroed before the launch) counts the CTAs that finished each block
  int ag_world, ag_rank, ag_rows, ag_seq;
  const void* ag_src[8];
  const int* ag_ready[8];
  int* ag_count;
  long long ag_spin;
};
int gemm_tc_launch(const GemmArgs& a, int sms, cudaStream_t st);
void gemm_tc_set_pair(int on);   // 1 (default): two-SM tcgen05 tiles, 0: one-SM tiles

// tensor-parallel row-parallel GEMM fused with its all-reduce over peer memory (tp_fused.cu)
#define TPF_MAXW 8
struct TpfArgs {
  const __nv_bfloat16* A;      // this rank's [M, K] activations (row-major)
  const __nv_bfloat16* Bt;     // this rank's projection rows, transposed: [N, K]
  int M, N, K;                 // M % 128 == 0, N % 128 == 0, K % 64 == 0
  __nv_bfloat16* recv[TPF_MAXW];// every rank's receive buffer [world][rows_own, N] bf16 (peer-mapped):
                               // slot r holds rank r's partial of the owner's row tiles
  long rows_own;               // rows per slot: ceil(M / 128 / world) * 128
  __nv_bfloat16* out[TPF_MAXW];// every rank's bf16 output [M, N] (peer-mapped)
  int* flags[TPF_MAXW];        // every rank's flag words [2][TPF_MAXW]
  int world, rank, seq;
  long long spin_limit;
  int* status;                 // 0 ok; 1 a GEMM-pipeline wait timed out; 2 a phase-3 copy wait timed out;
                               // 100 + phase a peer did not arrive
  int* abort;                  // zeroed before the launch
  unsigned long long* stamps;  // optional [4 + gridDim] %globaltimer stamps (ns): block 0 at launch, after
                               // the phase-1 grid barrier, after phase 3, at exit; then each CTA's end of
                               // phase-1 work (nullptr: none recorded)
};
int tp_gemm_allreduce_launch(const TpfArgs& a, int sms, cudaStream_t st);

// causal / sliding-window flash attention (attention.cu); strides in elements
struct AttnArgs {
  const __nv_bfloat16 *q, *k, *v;  // q [B, Lq, nh, HD], k/v [B, Lk, nh, HD] (strided)
  __nv_bfloat16* o;                // [B, Lq, nh, HD] (strided)
  float* lse;                      // [B, nh, Lq] base-2 log-sum-exp of the scaled scores
  long sq_b, sq_l, sq_h, sk_b, sk_l, sk_h, sv_b, sv_l, sv_h, so_b, so_l, so_h;
  int B, nh, Lq, Lk, q_offset, window;  // window <= 0: unbounded
  float scale_log2;                // softmax scale * log2(e)
  const int* kpos;                 // optional [B, Lk] absolute key positions (nullptr: the key index)
  const int* qoff;                 // optional [B] per-entry query offsets (nullptr: q_offset)
  int* status;                     // optional: set to 1 when a bounded wait of the tcgen05 forward timed out
  // optional block-indirect keys (NSA selection): entry b's key block j (64 keys) is rows
  // [64 kblk[b][j], 64 kblk[b][j] + 64) of source batch b / kb_ng of k / v; Lk = 64 kb_n
  const int* kblk;                 // [B, kb_n] int32, or nullptr (indices clamped to [0, kb_max])
  int kb_n, kb_ng, kb_max;
};
struct AttnBwdArgs {
  AttnArgs f;                      // the forward's tensors (o, lse as written by it)
  const __nv_bfloat16* dout;       // [B, Lq, nh, HD] (strided)
  long sd_b, sd_l, sd_h;
  float* D;                        // [B, nh, Lq] scratch: rowsum(dO * O)
  float* dq_acc;                   // [B, Lq, nh, HD] fp32, zeroed by the caller
  __nv_bfloat16 *dk, *dv;          // [B, Lk, nh, HD] (strided)
  long sdk_b, sdk_l, sdk_h, sdv_b, sdv_l, sdv_h;
  float scale;                     // softmax scale
  // with block-indirect keys: dK / dV are added (fp32 atomics) into the source-shaped,
  // contiguous [B / kb_ng, kb_lsrc, nh, HD] buffers instead of dk / dv
  float *dk_acc, *dv_acc;
  int kb_lsrc;
};
int attn_fwd_launch(const AttnArgs& a, int hd, cudaStream_t st);
int attn_bwd_launch(const AttnBwdArgs& a, int hd, cudaStream_t st);
// imp [B, Lq, Lk] = head-summed softmax probabilities of a finished forward (lse)
int attn_probsum_launch(const AttnArgs& a, float* imp, int hd, cudaStream_t st);

// cross-chunk state scan of the chunked gated delta rule (gdn_scan.cu); chunk length 64,
// value rows split in blocks of 64; every tensor contiguous
struct GdnArgs {
  const __nv_bfloat16 *qe, *kc, *kd;  // [B, nh, nc, 64, HD]
  const __nv_bfloat16* intra;         // [B, nh, nc, 64, 64] (lower triangle incl. diagonal)
  const float* vc;                    // [B, nh, nc, 64, HVD]
  const float* tot;                   // [B, nh, nc, HD] per-key-column decay over the chunk
  const float* S0;                    // [B, nh, HVD, HD] initial state (nullptr: zeros)
  float* o;                           // [B, nh, nc, 64, HVD]
  float* S_all;                       // [B, nh, nc, HVD, HD] state at each chunk start
  float* vnew;                        // [B, nh, nc, 64, HVD]
  float* S_fin;                       // [B, nh, HVD, HD]
  const float* dout;                  // backward: dL/do [B, nh, nc, 64, HVD]
  const float* dS_fin;                // backward: dL/dS_fin (nullptr: zeros)
  float *dqe_p, *dkc_p, *dkd_p;       // [HVD / VBb, B, nh, nc, 64, HD] per value-block partials
  float* din_p;                       // [HVD / VBb, B, nh, nc, 64, 64]
  float* dtot_p;                      // [HVD / VBb, B, nh, nc, HD]  (VBb = gdn_scan_bwd_value_block())
  float* dvc;                         // [B, nh, nc, 64, HVD]
  float* dS0;                         // [B, nh, HVD, HD]
  int B, nh, nc, HVD;
};
int gdn_scan_launch(const GdnArgs& a, int hd, bool bwd, int sms, cudaStream_t st);
int gdn_scan_bwd_value_block();

// intra-chunk score / WY matrices of the per-key-dim-decay delta rule (kda_intra.cu);
// N chunks of 64 steps, every tensor contiguous fp32
struct KdaArgs {
  const float *q, *k, *kb, *G;        // [N, 64, HD]; G = within-chunk cumulative log decay
  float *intra, *Lm;                  // forward outputs [N, 64, 64]
  const float *gI, *gL;               // backward inputs [N, 64, 64]
  float *dq, *dk, *dkb, *dG;          // backward outputs [N, 64, HD]
  long N;
  int HD;                             // a multiple of 32
};
int kda_intra_launch(const KdaArgs& a, bool bwd, cudaStream_t st);

// S5 complex diagonal recurrence x_t = lam * x_{t-1} + Bu_t (s5_scan.cu); complex64 as float2,
// every tensor contiguous, chunks of 64 steps
struct S5Args {
  const float2* lam;                  // [P]
  const float2* bu;                   // [B, L, P]
  const float2* x0;                   // [B, P] initial state (nullptr: zeros)
  float2* xs;                         // [B, L, P] (forward output; backward input)
  float2* xlast;                      // [B, P]
  float2* part;                       // [B, nchunk, P] scratch
  const float2* dxs;                  // backward: [B, L, P]
  const float2* dxlast;               // backward: [B, P] (nullptr: zeros)
  float2 *dbu, *dlam, *dx0;           // backward outputs ([B, L, P], [P] zeroed, [B, P] or nullptr)
  long B;
  int L, P, nchunk;
};
int s5_scan_launch(const S5Args& a, bool bwd, cudaStream_t st);

// recurrent decode step of the gated delta rule (gdn_decode.cu); fp32, contiguous
struct GdnDecodeArgs {
  const float *q, *k;                 // [B, T, nh, HD]
  const float* v;                     // [B, T, nh, hvd]
  const float* beta;                  // [B, T, nh]
  const float* alog;                  // [B, T, nh, alog_dim]  (alog_dim 1: per head, HD: per key dim)
  float* S;                           // [B, nh, hvd, HD] updated in place
  float* o;                           // [B, T, nh, hvd]
  int B, T, nh, hvd, alog_dim;
};
int gdn_decode_launch(const GdnDecodeArgs& a, int hd, cudaStream_t st);
