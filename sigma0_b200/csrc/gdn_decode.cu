// Recurrent (decode) step of the gated delta rule (GDN / KDA) for sm_100a.
//
// Per token t and head, with the state S [hvd, hd] (fp32, updated in place):
//   S <- S * alpha_t            (alpha = exp(alog): one value per head (GDN) or per key dim (KDA))
//   S <- S + beta_t (v_t - S k_t) k_t^T
//   o_t = S q_t
// (the reference's __call_rnn__, src/base_model/models/gdn.py:245-320).  The value rows of S
// are independent, so one warp owns one row: lane l holds key columns l, l + 32, ... in
// registers for all T tokens of the call, the two dot products are warp sums, and the state
// is read and written once per call -- a bandwidth-bound kernel like the Mamba3 decode step.
#include <cuda_runtime.h>

#include "launchers.h"

namespace s0 {
namespace gdn_dec {

constexpr int NW = 8;   // warps (value rows) per block

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int HD>
__global__ void __launch_bounds__(NW * 32) gdn_decode_k(GdnDecodeArgs a) {
  constexpr int PL = HD / 32;                       // key columns per lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * NW + warp;    // over B * nh * hvd
  const long rows = (long)a.B * a.nh * a.hvd;
  if (row >= rows) return;
  const int vr = (int)(row % a.hvd);
  const long bh = row / a.hvd;
  const int h = (int)(bh % a.nh), b = (int)(bh / a.nh);
  float* S = a.S + row * HD;
  float s[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) s[i] = S[lane + 32 * i];
  for (int t = 0; t < a.T; ++t) {
    const long tok = ((long)b * a.T + t) * a.nh + h;                  // (b, t, h)
    const float* q = a.q + tok * HD;
    const float* k = a.k + tok * HD;
    const float* al = a.alog + tok * a.alog_dim;
    const float beta = a.beta[tok];
    const float vv = a.v[tok * a.hvd + vr];
    float kk[PL], sk = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int d = lane + 32 * i;
      const float alpha = expf(a.alog_dim == 1 ? al[0] : al[d]);
      s[i] *= alpha;
      kk[i] = k[d];
      sk += s[i] * kk[i];
    }
    const float delta = beta * (vv - warp_sum(sk));
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      s[i] += delta * kk[i];
      sq += s[i] * q[lane + 32 * i];
    }
    sq = warp_sum(sq);
    if (lane == 0) a.o[tok * a.hvd + vr] = sq;
  }
#pragma unroll
  for (int i = 0; i < PL; ++i) S[lane + 32 * i] = s[i];
}

}  // namespace gdn_dec
}  // namespace s0

int gdn_decode_launch(const GdnDecodeArgs& a, int hd, cudaStream_t st) {
  using namespace s0::gdn_dec;
  const long rows = (long)a.B * a.nh * a.hvd;
  if (rows <= 0 || a.T <= 0) return 0;
  const unsigned grid = (unsigned)((rows + NW - 1) / NW);
  if (hd == 64) gdn_decode_k<64><<<grid, NW * 32, 0, st>>>(a);
  else if (hd == 128) gdn_decode_k<128><<<grid, NW * 32, 0, st>>>(a);
  else return -1;
  return (int)cudaGetLastError();
}
