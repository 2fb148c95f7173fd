// GDN pooled multi-token decode on a bf16 state pool, tensor-core form (sm_100a).
//
// Same contract as the multi-token bf16 path of gdn_decode_pool.cu (T tokens per
// sequence applied in order to the state read from pool slot in_slots[b] and
// written to out_slots[b]; the math per token is that of
// definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:91-132: s <- g s,
// delta = beta (v - k.s), s <- s + delta k, o = scale q.s), computed in closed
// form instead of token by token.  With C_t = g_0 ... g_t and
// D[t][tau] = g_{tau+1} ... g_t (D[t][t] = 1), every row s of the state obeys
//   d_t     = C_t (k_t . s_0) + sum_{tau<t} D[t][tau] (k_t . k_tau) delta_tau
//   delta_t = beta_t (v_t - d_t)
//   o_t     = scale (C_t (q_t . s_0) + sum_{tau<=t} D[t][tau] (q_t . k_tau) delta_tau)
//   s_T     = C_{T-1} s_0 + sum_tau D[T-1][tau] delta_tau k_tau,
// so a (sequence, v-head) needs only the 2T dot products of each state row with
// the tokens' k and q -- one tcgen05 MMA, S_0 [K;Q]^T (M = 128 rows, N = 2 TP,
// K = 128), whose bf16 operands are exact because the pool is bf16 -- a T x T
// triangular solve per row in fp32, and one rank-T update of the state in fp32.
// The per-token form spends four multiply-adds per state element and token on
// CUDA cores; this one spends T + 1 per element for all T tokens.
//
// One CTA per (sequence, v-head), 256 threads:
//   * thread 0 loads the 32 KiB state tile and the T k and q rows by TMA
//     (128-byte swizzle) and issues the MMA (D in TMEM, 2 TP columns);
//   * every octet of lanes forms the tokens' Gram products (k_t . k_tau,
//     q_t . k_tau, and |q_t|^2 / |k_t|^2 for the optional L2 norm) from the
//     token tile, and warp 0 the per-head tables (gates, decay products);
//   * warps 0-3 (thread = state row) read their row's 2T dot products from TMEM,
//     solve for delta, write the T outputs and the row's update weights;
//   * all eight warps form s_T = C s_0 + sum_tau w_tau k_tau from the state tile in
//     shared memory (16-byte chunks, two full rows per warp instruction) and
//     stream it to the pool.
// q/k L2 normalisation (x / sqrt(sum x^2 + 1e-6)) is applied as per-token factors
// on the dot products and the update weights; q and k themselves are never
// rescaled, so the MMA operands stay exact.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_sm100.cuh"

namespace gdn {

// Status word of this translation unit (bit kStatusPoolTimeout), merged into the
// library's word by read_status.
__device__ uint32_t g_pool_tc_status = 0;

namespace {
using namespace sm100;

constexpr int kThreads = 256;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kStateBytes = kHead * kHead * 2;  // one bf16 state tile
constexpr uint32_t kKb = 16384;                      // one 64-column block of the state tile

__device__ __forceinline__ void st_stream_u4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Shared-memory layout for a token count bound TP (8, 16, 24 or 32); T <= TP.
template <int TP>
struct PoolTcLayout {
  static constexpr int N1 = 2 * TP;                           // MMA N: k rows [0,TP), q rows [TP,2TP)
  static constexpr uint32_t kTokKb = N1 * 128;                // one 64-column block of the token tile
  static constexpr uint32_t OFF_S = 0;                        // state tile [kb 2][128][128 B]
  static constexpr uint32_t OFF_TOK = OFF_S + kStateBytes;    // token tile [kb 2][N1][128 B]
  static constexpr uint32_t OFF_G = OFF_TOK + 2 * kTokKb;     // Gram: KK[TP][TP], QK[TP][TP], QQ[TP]
  static constexpr uint32_t OFF_TAB = OFF_G + (2 * TP * TP + TP) * 4;
  // tables: Ak[TP][TP], Bq[TP][TP], Ck[TP], Cq[TP], beta[TP], w[TP], g[TP], C_final
  static constexpr uint32_t OFF_W = OFF_TAB + (2 * TP * TP + 5 * TP + 4) * 4;  // weights [128][TP]
  static constexpr uint32_t OFF_BAR = OFF_W + 128 * TP * 4;
  static constexpr uint32_t kBytes = OFF_BAR + 64 + 1024;     // + barriers, slack for 1024 alignment
  static constexpr uint32_t kTmemCols = N1 <= 32 ? 32 : 64;
};

template <int TP, bool L2NORM>
__global__ void __launch_bounds__(kThreads, TP <= 8 ? 4 : (TP <= 16 ? 2 : 1))
    gdn_decode_pool_tc_kernel(const __grid_constant__ CUtensorMap tm_pool,
                              const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k, DecodePoolArgs p) {
  using Lay = PoolTcLayout<TP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  float* G = reinterpret_cast<float*>(smem + Lay::OFF_G);
  float* KK = G;
  float* QK = G + TP * TP;
  float* QQ = G + 2 * TP * TP;
  float* tab = reinterpret_cast<float*>(smem + Lay::OFF_TAB);
  float* Ak = tab;                 // D[t][tau] (k^_t . k^_tau), tau < t
  float* Bq = Ak + TP * TP;        // scale D[t][tau] (q^_t . k^_tau), tau <= t
  float* Ck = Bq + TP * TP;        // C_t / |k_t|
  float* Cq = Ck + TP;             // scale C_t / |q_t|
  float* bet = Cq + TP;            // beta_t
  float* wgt = bet + TP;           // D[T-1][tau] / |k_tau|: weight of delta_tau k_tau in s_T
  float* gg = wgt + TP;            // g_t
  float* cfin = gg + TP;           // C_{T-1}
  float* W = reinterpret_cast<float*>(smem + Lay::OFF_W);  // per row: w_tau delta_tau
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::OFF_BAR);  // 0: TMA, 1: MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = static_cast<int>(p.T);
  const int64_t bh = blockIdx.x;  // b * Hv + h
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);
  const int32_t sin = p.in_slots[bidx];
  const int32_t sout = p.out_slots ? p.out_slots[bidx] : sin;
  const bool has_in = sin >= 0 && sin < p.pool_size;
  const bool write_back = !p.no_state_update && sout >= 0 && sout < p.pool_size;

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    if (has_in) prefetch_tmap(&tm_pool);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Lay::kTmemCols);
    tmem_relinquish();
  }
  if (!has_in) {  // zero initial state: an all-zero tile (read by the MMA and the update)
    for (uint32_t i = tid; i < kStateBytes / 16; i += kThreads) sts128(sb + Lay::OFF_S + 16 * i, 0u, 0u, 0u, 0u);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool failed = false;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], (has_in ? kStateBytes : 0u) + 4u * T * 128u);
    if (has_in) {
      const int tile = static_cast<int>(static_cast<int64_t>(sin) * p.Hv + h);
      tma_load_3d(smem + Lay::OFF_S, &tm_pool, &bars[0], 0, 0, tile);
      tma_load_3d(smem + Lay::OFF_S + kKb, &tm_pool, &bars[0], 64, 0, tile);
    }
    const int tok = static_cast<int>(bidx * p.T);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_3d(smem + Lay::OFF_TOK + kb * Lay::kTokKb, &tm_k, &bars[0], kb * 64, qh, tok);
      tma_load_3d(smem + Lay::OFF_TOK + kb * Lay::kTokKb + TP * 128, &tm_q, &bars[0], kb * 64, qh, tok);
    }
  }
  // gates of the T tokens (warp 1, lane t), independent of the loads
  if (warp == 1 && lane < T) {
    const int64_t bt = bidx * p.T + lane;
    const float a = __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[bt * p.Hv + h]);
    const float b = __bfloat162float(static_cast<const __nv_bfloat16*>(p.b)[bt * p.Hv + h]);
    gg[lane] = expf(log_decay(p.A_log[h], a, p.dt_bias[h]));
    bet[lane] = sigmoidf_acc(b);
  }
  // this row's v values (warps 0-3: thread = state row), in flight during the wait
  float vrow[TP];
  if (warp < 4) {
    const __nv_bfloat16* vp = static_cast<const __nv_bfloat16*>(p.v) + (bidx * p.T * p.Hv + h) * kHead + tid;
#pragma unroll
    for (int t = 0; t < TP; ++t) vrow[t] = t < T ? __bfloat162float(vp[static_cast<int64_t>(t) * p.Hv * kHead]) : 0.f;
  }

  if (!mbar_wait(&bars[0], 0, kTimeoutNs)) failed = true;
  if (tid == 0 && !failed) {  // S_0 [K;Q]^T -> TMEM columns [0, 2 TP)
    tc_fence_after();
    const uint32_t idesc = idesc_bf16(128, Lay::N1, false, false);
    const uint32_t s16 = (sb + Lay::OFF_S) >> 4, t16 = (sb + Lay::OFF_TOK) >> 4;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint64_t a = sdesc_sw128_f(s16 + ((ks >> 2) * kKb + (ks & 3) * 32) / 16, 16, 1024);
      const uint64_t b = sdesc_sw128_f(t16 + ((ks >> 2) * Lay::kTokKb + (ks & 3) * 32) / 16, 16, 1024);
      mma_bf16_ss(tmem, a, b, idesc, ks > 0);
    }
    mma_commit(&bars[1]);
  }

  // Gram products of the tokens, one octet per product pair: task (t, tau) with
  // tau <= t gives k_t . k_tau and q_t . k_tau; with the L2 norm, T more tasks
  // give q_t . q_t.  Lane j of the octet takes 16-byte chunk j of both 64-column
  // blocks of each row.
  {
    const int oct = tid >> 3, j = tid & 7;
    const int ntri = T * (T + 1) / 2;
    const int ntask = ntri + (L2NORM ? T : 0);
    const uint32_t tok = sb + Lay::OFF_TOK;
    for (int base = 0; base < ntask; base += kThreads / 8) {
      const int task = base + oct;
      int t = 0, tau = 0;
      bool qq = false;
      if (task < ntri) {
        while ((t + 1) * (t + 2) / 2 <= task) ++t;
        tau = task - t * (t + 1) / 2;
      } else {
        qq = true;
        t = tau = min(task - ntri, T - 1);
      }
      float d0 = 0.f, d1 = 0.f;
      if (task < ntask && !failed) {
        const int r0 = qq ? TP + t : t;  // k_t (or q_t)
        const int r2 = qq ? TP + t : tau;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t blk = tok + kb * Lay::kTokKb;
          const uint4 x = lds128(blk + sw128_off(r0, j));
          const uint4 y = lds128(blk + sw128_off(TP + t, j));
          const uint4 z = lds128(blk + sw128_off(r2, j));
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w},
                         zs[4] = {z.x, z.y, z.z, z.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            d0 = fmaf(bf16_lo(xs[e]), bf16_lo(zs[e]), fmaf(bf16_hi(xs[e]), bf16_hi(zs[e]), d0));
            d1 = fmaf(bf16_lo(ys[e]), bf16_lo(zs[e]), fmaf(bf16_hi(ys[e]), bf16_hi(zs[e]), d1));
          }
        }
      }
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        d0 += __shfl_xor_sync(0xffffffffu, d0, m);
        d1 += __shfl_xor_sync(0xffffffffu, d1, m);
      }
      if (j == 0 && task < ntask) {
        if (qq) {
          QQ[t] = d0;
        } else {
          KK[t * TP + tau] = d0;
          QK[t * TP + tau] = d1;
        }
      }
    }
  }
  __syncthreads();

  // per-head tables (warp 0, lane t)
  if (warp == 0) {
    const int t = lane;
    if (t < T) {
      const float rk_t = L2NORM ? rsqrtf(KK[t * TP + t] + 1e-6f) : 1.f;
      const float rq_t = L2NORM ? rsqrtf(QQ[t] + 1e-6f) : 1.f;
      // C_t and D[t][tau] as running products of the gates (as the token loop
      // multiplies the state by each g in turn)
      float c = 1.f;
      for (int s = 0; s <= t; ++s) c *= gg[s];
      Ck[t] = c * rk_t;
      Cq[t] = p.scale * c * rq_t;
      float d = 1.f;  // D[t][tau], tau = t, t-1, ..., 0
      for (int tau = t; tau >= 0; --tau) {
        const float rk_tau = L2NORM ? rsqrtf(KK[tau * TP + tau] + 1e-6f) : 1.f;
        Ak[t * TP + tau] = tau < t ? d * rk_t * rk_tau * KK[t * TP + tau] : 0.f;
        Bq[t * TP + tau] = p.scale * d * rq_t * rk_tau * QK[t * TP + tau];
        if (tau > 0) d *= gg[tau];
      }
      float dw = 1.f;  // D[T-1][t]
      for (int s = t + 1; s < T; ++s) dw *= gg[s];
      wgt[t] = dw * rk_t;
      if (t == T - 1) *cfin = c;
    }
  }
  __syncthreads();

  // warps 0-3: thread = state row; its 2T dot products from TMEM, the solve, the
  // outputs and the row's update weights
  if (warp < 4) {
    if (!failed && !mbar_wait(&bars[1], 0, kTimeoutNs)) failed = true;
    tc_fence_after();
    float dk[Lay::N1];
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
    for (int c0 = 0; c0 < Lay::N1; c0 += 16) tmem_ld16(taddr + c0, dk + c0);
    tmem_wait_ld();
    reg_fence(dk);
    float delta[TP];
    __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) + (bidx * p.T * p.Hv + h) * kHead + tid;
#pragma unroll
    for (int t = 0; t < TP; ++t) {
      if (t < T) {
        float dt = Ck[t] * dk[t];
        float o = Cq[t] * dk[TP + t];
#pragma unroll
        for (int tau = 0; tau < t; ++tau) {
          dt = fmaf(Ak[t * TP + tau], delta[tau], dt);
          o = fmaf(Bq[t * TP + tau], delta[tau], o);
        }
        delta[t] = bet[t] * (vrow[t] - dt);
        o = fmaf(Bq[t * TP + t], delta[t], o);
        op[static_cast<int64_t>(t) * p.Hv * kHead] = __float2bfloat16_rn(o);
      } else {
        delta[t] = 0.f;
      }
    }
    float* wr = W + tid * TP;
#pragma unroll
    for (int t = 0; t < TP; t += 4)
      *reinterpret_cast<float4*>(wr + t) =
          make_float4(wgt[t] * delta[t], t + 1 < T ? wgt[t + 1] * delta[t + 1] : 0.f,
                      t + 2 < T ? wgt[t + 2] * delta[t + 2] : 0.f, t + 3 < T ? wgt[t + 3] * delta[t + 3] : 0.f);
  }
  __syncthreads();

  // all warps: s_T = C_{T-1} s_0 + sum_tau w_tau k_tau, 16-byte chunks; a warp
  // instruction covers two full rows (512 contiguous bytes of the pool)
  if (write_back && !failed) {
    const float cf = *cfin;
    const int kc = lane & 15, kb = kc >> 3, c = kc & 7;
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.pool) +
                         (static_cast<int64_t>(sout) * p.Hv + h) * (kHead * kHead) + 8 * kc;
    const uint32_t sblk = sb + Lay::OFF_S + kb * kKb;
    const uint32_t tblk = sb + Lay::OFF_TOK + kb * Lay::kTokKb;
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int row = 16 * warp + 2 * i + (lane >> 4);
      const uint4 s4 = lds128(sblk + sw128_off(row, c));
      const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
      float x[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 r = __fmul2_rn(make_float2(bf16_lo(sw[e]), bf16_hi(sw[e])), make_float2(cf, cf));
        x[2 * e] = r.x;
        x[2 * e + 1] = r.y;
      }
      const float* wr = W + row * TP;
#pragma unroll 4
      for (int tau = 0; tau < T; ++tau) {
        const float w = wr[tau];
        const uint4 k4 = lds128(tblk + sw128_off(tau, c));
        const uint32_t kw[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 r = __ffma2_rn(make_float2(bf16_lo(kw[e]), bf16_hi(kw[e])), make_float2(w, w),
                                      make_float2(x[2 * e], x[2 * e + 1]));
          x[2 * e] = r.x;
          x[2 * e + 1] = r.y;
        }
      }
      st_stream_u4(dst + static_cast<int64_t>(row) * kHead,
                   make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                              pack_bf16x2(x[6], x[7])));
    }
  }
  if (failed) atomicOr(&g_pool_tc_status, kStatusPoolTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, Lay::kTmemCols);
  }
}

// [rows, 128] bf16 views used by the kernel: the pool as [P*Hv tiles][128][128]
// (box = one 64-column block of a whole tile) and q/k as [B*T][H][128] (box = T
// token rows of one head, 64 columns); 128-byte swizzle throughout.
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

cudaError_t encode_map(CUtensorMap* m, const void* base, uint64_t d1, uint64_t d2, uint32_t b1,
                       uint32_t b2) {
  auto fn = encoder();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHead), d1, d2};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHead) * 2, static_cast<cuuint64_t>(d1) * kHead * 2};
  cuuint32_t box[3] = {64, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int TP>
cudaError_t launch_tp(const DecodePoolArgs& a, cudaStream_t s) {
  using Lay = PoolTcLayout<TP>;
  CUtensorMap mp, mq, mk;
  memset(&mp, 0, sizeof(mp));
  cudaError_t e;
  if ((e = encode_map(&mp, a.pool, kHead, static_cast<uint64_t>(a.pool_size * a.Hv), 128, 1)) != cudaSuccess)
    return e;
  if ((e = encode_map(&mq, a.q, a.Hq, static_cast<uint64_t>(a.B * a.T), 1, static_cast<uint32_t>(a.T))) !=
      cudaSuccess)
    return e;
  if ((e = encode_map(&mk, a.k, a.Hq, static_cast<uint64_t>(a.B * a.T), 1, static_cast<uint32_t>(a.T))) !=
      cudaSuccess)
    return e;
  auto kernel = a.qk_l2norm ? gdn_decode_pool_tc_kernel<TP, true> : gdn_decode_pool_tc_kernel<TP, false>;
  if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), Lay::kBytes)) != cudaSuccess) return e;
  const int64_t ctas = a.B * a.Hv;
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  kernel<<<static_cast<unsigned>(ctas), kThreads, Lay::kBytes, s>>>(mp, mq, mk, a);
  return cudaGetLastError();
}

}  // namespace

bool decode_pool_tc_supported(const DecodePoolArgs& a) {
  // bf16 pool, 2..32 tokens, no per-token state cache; TMA needs 16-byte aligned
  // bases (the pool tile rows, q and k rows are 256-byte multiples beyond that)
  return a.state_bf16 && a.T >= 2 && a.T <= 32 && a.intermediate == nullptr && a.pool_size > 0 &&
         reinterpret_cast<uintptr_t>(a.pool) % 16 == 0 && reinterpret_cast<uintptr_t>(a.q) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.k) % 16 == 0 && a.pool_size * a.Hv <= 0x7fffffffLL &&
         a.B * a.T <= 0x7fffffffLL;
}

cudaError_t read_pool_tc_status(uint32_t* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_pool_tc_status, sizeof(uint32_t));
  if (e != cudaSuccess || !clear) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_pool_tc_status, &zero, sizeof(uint32_t));
}

cudaError_t launch_decode_pool_tc(const DecodePoolArgs& a, cudaStream_t s) {
  if (a.T <= 8) return launch_tp<8>(a, s);
  if (a.T <= 16) return launch_tp<16>(a, s);
  if (a.T <= 24) return launch_tp<24>(a, s);
  return launch_tp<32>(a, s);
}

}  // namespace gdn
