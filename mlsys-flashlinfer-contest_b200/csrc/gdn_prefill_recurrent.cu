// GDN prefill, token-recurrent form on CUDA cores (sm_100a).
//
// Replaces gdn_prefill/solution/python/cuda_recurrent_v1.cu:128-222 (the
// reference's path for tiny prefill workloads, chosen at
// gdn_prefill/solution/python/gdn_prefill_mix.py:29).  Same row decomposition
// as the decode kernel: an aligned octet of 8 lanes owns one state row
// S[v][0..127] for the whole sequence, the row stays in registers across tokens,
// and it is written to new_state once at the end.  The next token's q/k/v/a/b
// are fetched while the current token is processed.
//
// With qk_l2norm, q and k are L2-normalised per head first (x / sqrt(sum x^2 + 1e-6)).
// Semantics follow definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:108-142:
// state == nullptr means a zero initial state, and a sequence of length 0 ends
// with a zero final state (the definition skips it and new_state starts at 0).
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kThreads = 128;           // 4 warps, 16 rows per CTA
constexpr int kRowsPerCta = 16;
constexpr int kTilesPerHead = kHead / kRowsPerCta;

struct TokenIn {
  float k[16], q[16];
  float v, a, b;
};

__device__ __forceinline__ void load_token(const PrefillArgs& p, int64_t t, int h, int qh, int row,
                                           int j, TokenIn& in) {
  const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(p.k) + (t * p.Hq + qh) * kHead;
  const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(p.q) + (t * p.Hq + qh) * kHead;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ld_bf16x4(kp + 32 * i + 4 * j, in.k + 4 * i);
    ld_bf16x4(qp + 32 * i + 4 * j, in.q + 4 * i);
  }
  const int64_t th = t * p.Hv + h;
  in.v = __bfloat162float(static_cast<const __nv_bfloat16*>(p.v)[th * kHead + row]);
  in.a = __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[th]);
  in.b = __bfloat162float(static_cast<const __nv_bfloat16*>(p.b)[th]);
}

__global__ void __launch_bounds__(kThreads) gdn_prefill_recurrent_kernel(PrefillArgs p) {
  const int64_t cta = blockIdx.x;
  const int64_t nh = cta / kTilesPerHead;  // n * Hv + h
  const int tile = static_cast<int>(cta % kTilesPerHead);
  const int64_t n = nh / p.Hv;
  const int h = static_cast<int>(nh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = lane & 7;
  const int row = tile * kRowsPerCta + warp * 4 + (lane >> 3);

  // cu_seqlens is caller data read only here: clamp it into [0, T] so a bad
  // value can never move an access outside the packed tensors.
  const int64_t t0 = min(max(p.cu_seqlens[n], int64_t(0)), p.T);
  const int64_t t1 = min(max(p.cu_seqlens[n + 1], t0), p.T);
  const int64_t row_elem = (nh * kHead + row) * kHead + 4 * j;

  float S[16];
  if (p.state != nullptr && t1 > t0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 x = ld_stream_f4(p.state + row_elem + 32 * i);
      S[4 * i + 0] = x.x;
      S[4 * i + 1] = x.y;
      S[4 * i + 2] = x.z;
      S[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 16; ++c) S[c] = 0.0f;
  }

  const float A_log = p.A_log[h], dt_bias = p.dt_bias[h];
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
  TokenIn cur, nxt;
  if (t0 < t1) load_token(p, t0, h, qh, row, j, cur);
  for (int64_t t = t0; t < t1; ++t) {
    if (t + 1 < t1) load_token(p, t + 1, h, qh, row, j, nxt);
    const float g = expf(log_decay(A_log, cur.a, dt_bias));
    const float beta = sigmoidf_acc(cur.b);
    if (p.qk_l2norm) {  // x / sqrt(sum x^2 + 1e-6), the sum over the octet
      float sk = 0.0f, sq = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        sk = fmaf(cur.k[c], cur.k[c], sk);
        sq = fmaf(cur.q[c], cur.q[c], sq);
      }
      const float rk = rsqrtf(octet_sum(sk) + 1e-6f), rq = rsqrtf(octet_sum(sq) + 1e-6f);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        cur.k[c] *= rk;
        cur.q[c] *= rq;
      }
    }
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      S[c] *= g;
      dot = fmaf(cur.k[c], S[c], dot);
    }
    dot = octet_sum(dot);
    const float delta = beta * (cur.v - dot);
    float ov = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      S[c] = fmaf(cur.k[c], delta, S[c]);
      ov = fmaf(cur.q[c], S[c], ov);
    }
    ov = octet_sum(ov);
    if (j == 0) out[(t * p.Hv + h) * kHead + row] = __float2bfloat16_rn(p.scale * ov);
    cur = nxt;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    st_stream_f4(p.new_state + row_elem + 32 * i,
                 make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]));
}

}  // namespace

cudaError_t launch_prefill_recurrent(const PrefillArgs& a, cudaStream_t s) {
  if (a.N == 0) return cudaSuccess;
  const int64_t ctas = a.N * a.Hv * kTilesPerHead;
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  gdn_prefill_recurrent_kernel<<<static_cast<unsigned>(ctas), kThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace gdn
