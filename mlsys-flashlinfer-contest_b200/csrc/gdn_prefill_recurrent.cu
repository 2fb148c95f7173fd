// GDN prefill, token-recurrent form on CUDA cores (sm_100a).
//
// Replaces gdn_prefill/solution/python/cuda_recurrent_v1.cu:128-222 (the
// reference's path for tiny prefill workloads, chosen at
// gdn_prefill/solution/python/gdn_prefill_mix.py:29).  Same row decomposition
// as the decode kernel: an aligned octet of 8 lanes owns one state row
// S[v][0..127] for the whole sequence, the row stays in registers across tokens,
// and it is written to new_state once at the end.  Tokens pass through shared
// memory in blocks of 16, the next block copied while the current one is applied.
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
constexpr int kTokBlock = 16;           // tokens staged in shared memory at a time

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// L2: q/k L2 norm (a separate instantiation, so the plain token loop carries no test).
template <bool L2>
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
  const __nv_bfloat16* kg = static_cast<const __nv_bfloat16*>(p.k);
  const __nv_bfloat16* qg = static_cast<const __nv_bfloat16*>(p.q);
  const __nv_bfloat16* vg = static_cast<const __nv_bfloat16*>(p.v);
  const __nv_bfloat16* ag = static_cast<const __nv_bfloat16*>(p.a);
  const __nv_bfloat16* bg = static_cast<const __nv_bfloat16*>(p.b);
  // Tokens go through shared memory in blocks of kTokBlock, double-buffered: the
  // next block's k, q (whole vectors) and this CTA's 16 v values per token are
  // copied asynchronously (cp.async) while the current block is applied, and its
  // gates are loaded into registers then, turned into (g, beta) after the block.
  __shared__ __align__(16) __nv_bfloat16 kq_s[2][kTokBlock][2 * kHead];  // k | q
  __shared__ __align__(16) __nv_bfloat16 v_s[2][kTokBlock][kRowsPerCta];
  __shared__ float gb_s[2][kTokBlock][2];
  const int tid = threadIdx.x;
  float ga_raw = 0.f, gb_raw = 0.f;  // gate inputs of token (block start + tid), tid < kTokBlock
  auto stage = [&](int buf, int64_t tb) {
    for (int i = tid; i < kTokBlock * 32; i += kThreads) {  // 16-byte pieces: 16 of k, 16 of q
      const int u = i >> 5, part = i & 31;
      const int64_t t = tb + u;
      if (t < t1) {
        const __nv_bfloat16* src = (part < 16 ? kg : qg) + (t * p.Hq + qh) * kHead + 8 * (part & 15);
        cp_async16(&kq_s[buf][u][8 * part], src);
      }
    }
    for (int i = tid; i < kTokBlock * 2; i += kThreads) {  // this CTA's 16 v values: 2 x 16 bytes
      const int u = i >> 1, half = i & 1;
      const int64_t t = tb + u;
      if (t < t1) cp_async16(&v_s[buf][u][8 * half], vg + (t * p.Hv + h) * kHead + tile * kRowsPerCta + 8 * half);
    }
    cp_async_commit();
    if (tid < kTokBlock && tb + tid < t1) {
      ga_raw = __bfloat162float(ag[(tb + tid) * p.Hv + h]);
      gb_raw = __bfloat162float(bg[(tb + tid) * p.Hv + h]);
    }
  };
  auto finish_stage = [&](int buf) {  // gates of the staged block, then wait for its copies
    if (tid < kTokBlock) {
      gb_s[buf][tid][0] = expf(log_decay(A_log, ga_raw, dt_bias));
      gb_s[buf][tid][1] = sigmoidf_acc(gb_raw);
    }
    cp_async_wait_all();
  };
  if (t0 < t1) {
    stage(0, t0);
    finish_stage(0);
  }
  __syncthreads();
  const int r_in = warp * 4 + (lane >> 3);  // this thread's row within the CTA's 16
  for (int64_t tb = t0, blk = 0; tb < t1; tb += kTokBlock, ++blk) {
    const int buf = static_cast<int>(blk & 1);
    const bool more = tb + kTokBlock < t1;
    if (more) stage(buf ^ 1, tb + kTokBlock);
    const int nt = static_cast<int>(min(static_cast<int64_t>(kTokBlock), t1 - tb));
    for (int u = 0; u < nt; ++u) {
      float kf[16], qf[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint2 wk = *reinterpret_cast<const uint2*>(&kq_s[buf][u][32 * i + 4 * j]);
        const uint2 wq = *reinterpret_cast<const uint2*>(&kq_s[buf][u][kHead + 32 * i + 4 * j]);
        kf[4 * i + 0] = bf16_lo(wk.x);
        kf[4 * i + 1] = bf16_hi(wk.x);
        kf[4 * i + 2] = bf16_lo(wk.y);
        kf[4 * i + 3] = bf16_hi(wk.y);
        qf[4 * i + 0] = bf16_lo(wq.x);
        qf[4 * i + 1] = bf16_hi(wq.x);
        qf[4 * i + 2] = bf16_lo(wq.y);
        qf[4 * i + 3] = bf16_hi(wq.y);
      }
      const float g = gb_s[buf][u][0], beta = gb_s[buf][u][1];
      const float vv = __bfloat162float(v_s[buf][u][r_in]);
      if constexpr (L2) {  // x / sqrt(sum x^2 + 1e-6), the sum over the octet
        float sk = 0.0f, sq = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          sk = fmaf(kf[c], kf[c], sk);
          sq = fmaf(qf[c], qf[c], sq);
        }
        const float rk = rsqrtf(octet_sum(sk) + 1e-6f), rq = rsqrtf(octet_sum(sq) + 1e-6f);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          kf[c] *= rk;
          qf[c] *= rq;
        }
      }
      // element pairs on the packed FMUL2 / FFMA2 path (each lane rounds like the
      // scalar operation): two partial sums per dot product, half the chain
      float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        const float2 sv = __fmul2_rn(make_float2(S[c], S[c + 1]), make_float2(g, g));
        S[c] = sv.x;
        S[c + 1] = sv.y;
        d2 = __ffma2_rn(make_float2(kf[c], kf[c + 1]), sv, d2);
      }
      const float dot = octet_sum(d2.x + d2.y);
      const float delta = beta * (vv - dot);
      float2 o2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        const float2 sv = __ffma2_rn(make_float2(kf[c], kf[c + 1]), make_float2(delta, delta),
                                     make_float2(S[c], S[c + 1]));
        S[c] = sv.x;
        S[c + 1] = sv.y;
        o2 = __ffma2_rn(make_float2(qf[c], qf[c + 1]), sv, o2);
      }
      const float ov = octet_sum(o2.x + o2.y);
      if (j == 0) out[((tb + u) * p.Hv + h) * kHead + row] = __float2bfloat16_rn(p.scale * ov);
    }
    if (more) finish_stage(buf ^ 1);
    __syncthreads();
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
  if (a.qk_l2norm)
    gdn_prefill_recurrent_kernel<true><<<static_cast<unsigned>(ctas), kThreads, 0, s>>>(a);
  else
    gdn_prefill_recurrent_kernel<false><<<static_cast<unsigned>(ctas), kThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace gdn
