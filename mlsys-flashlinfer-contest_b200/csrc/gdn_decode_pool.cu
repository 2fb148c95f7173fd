// GDN pooled multi-token decode (serving form), sm_100a.
//
// The reference workspace decodes one token per sequence with a dense fp32 state
// batch (gdn_decode_final.py:23-36).  Serving stacks add three things around the
// same recurrence, and this kernel carries them in one pass over the state:
//   * a state pool: sequence b reads slot in_slots[b] of a [pool, Hv, 128, 128]
//     pool and writes slot out_slots[b] (in place when they match); a negative or
//     out-of-range read slot means a zero initial state, such a write slot means
//     no write-back;
//   * T >= 1 tokens per sequence applied in order (multi-token / speculative
//     decode), the state held in registers between tokens, optionally with the
//     state after every token written to a [B, T, Hv, 128, 128] cache;
//   * fp32 or bf16 state storage (bf16 halves the HBM bytes of the stream; the
//     arithmetic stays fp32 and the state is rounded once per store), and an
//     optional L2 normalisation of q and k per head inside the kernel
//     (x / sqrt(sum x^2 + 1e-6)).
// Per token the math is that of definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:91-132
// (as in gdn_decode.cu): g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b),
// old_v = k . (g S[v]), S'[v] = g S[v] + beta k (v[v] - old_v), o[v] = scale q . S'[v].
//
// Mapping: a CTA of 256 threads owns 32*U consecutive state rows of one (b, h);
// each aligned octet of 8 lanes owns one row at a time.  Lane j of the octet holds
// 16 of the row's elements such that every 16-byte load of the octet covers one
// contiguous 128-byte segment: k = 32 i + 4 j + c (i < 4, c < 4) for fp32 storage,
// k = 64 i + 8 j + c (i < 2, c < 8) for bf16; q and k are read in the same
// pattern.  All state loads of a thread are issued before any use, and the
// inputs of token t+1 are loaded while token t is applied.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cs.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_stream_u4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// This lane's 16 elements of a bf16 vector of 128 (q or k), widened to fp32, in
// the lane pattern of the state storage (see the mapping above).
template <bool BF16>
__device__ __forceinline__ void ld_vec16(const __nv_bfloat16* row, int j, float* out) {
  if constexpr (BF16) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 w;
      asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                   : "l"(row + 64 * i + 8 * j));
      out[8 * i + 0] = bf16_lo(w.x);
      out[8 * i + 1] = bf16_hi(w.x);
      out[8 * i + 2] = bf16_lo(w.y);
      out[8 * i + 3] = bf16_hi(w.y);
      out[8 * i + 4] = bf16_lo(w.z);
      out[8 * i + 5] = bf16_hi(w.z);
      out[8 * i + 6] = bf16_lo(w.w);
      out[8 * i + 7] = bf16_hi(w.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) ld_bf16x4(row + 32 * i + 4 * j, out + 4 * i);
  }
}

// One lane's 16 state elements of a row (row start at element offset `elem`):
// load from / store to fp32 or bf16 storage.
template <bool BF16>
__device__ __forceinline__ void load_row16(const void* base, int64_t elem, int j, float* s) {
  if constexpr (BF16) {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(base) + elem + 8 * j;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 w = ld_stream_u4(p + 64 * h);
      s[8 * h + 0] = bf16_lo(w.x);
      s[8 * h + 1] = bf16_hi(w.x);
      s[8 * h + 2] = bf16_lo(w.y);
      s[8 * h + 3] = bf16_hi(w.y);
      s[8 * h + 4] = bf16_lo(w.z);
      s[8 * h + 5] = bf16_hi(w.z);
      s[8 * h + 6] = bf16_lo(w.w);
      s[8 * h + 7] = bf16_hi(w.w);
    }
  } else {
    const float* p = static_cast<const float*>(base) + elem + 4 * j;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 x = ld_stream_f4(p + 32 * i);
      s[4 * i + 0] = x.x;
      s[4 * i + 1] = x.y;
      s[4 * i + 2] = x.z;
      s[4 * i + 3] = x.w;
    }
  }
}

template <bool BF16>
__device__ __forceinline__ void store_row16(void* base, int64_t elem, int j, const float* s) {
  if constexpr (BF16) {
    __nv_bfloat16* p = static_cast<__nv_bfloat16*>(base) + elem + 8 * j;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      st_stream_u4(p + 64 * h, make_uint4(pack_bf16x2(s[8 * h + 0], s[8 * h + 1]),
                                         pack_bf16x2(s[8 * h + 2], s[8 * h + 3]),
                                         pack_bf16x2(s[8 * h + 4], s[8 * h + 5]),
                                         pack_bf16x2(s[8 * h + 6], s[8 * h + 7])));
  } else {
    float* p = static_cast<float*>(base) + elem + 4 * j;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      st_stream_f4(p + 32 * i, make_float4(s[4 * i + 0], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]));
  }
}

// MTP: T > 1 (the next token's inputs are prefetched); two CTAs per SM keep the
// slot lookup, a dependent load in front of every state stream, overlapped.
// INTER: the per-token state cache may be written (multi-token instantiations
// without it carry no test per row and token: 5 % at T = 4).
template <int U, bool BF16, bool L2NORM, bool MTP, bool INTER = true>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_pool_kernel(DecodePoolArgs p) {
  constexpr int kRows = 32 * U;
  constexpr int kTilesPerHead = kHead / kRows;
  const int64_t cta = blockIdx.x;
  const int64_t bh = cta / kTilesPerHead;  // b * Hv + h
  const int tile = static_cast<int>(cta % kTilesPerHead);
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int oct = lane >> 3;
  const int j = lane & 7;
  const int row0 = tile * kRows + warp * (4 * U) + oct;  // rows row0 + 4u
  constexpr int64_t kTile = kHead * kHead;

  const int32_t sin = p.in_slots[bidx];
  const int32_t sout = p.out_slots ? p.out_slots[bidx] : sin;
  const bool has_in = sin >= 0 && sin < p.pool_size;
  const bool write_back = !p.no_state_update && sout >= 0 && sout < p.pool_size;

  float s[U][16];
  if (has_in) {
    const int64_t base = (static_cast<int64_t>(sin) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead;
#pragma unroll
    for (int u = 0; u < U; ++u) load_row16<BF16>(p.pool, base + u * 4 * kHead, j, s[u]);
  } else {
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int c = 0; c < 16; ++c) s[u][c] = 0.0f;
  }

  const __nv_bfloat16* a_ptr = static_cast<const __nv_bfloat16*>(p.a);
  const __nv_bfloat16* b_ptr = static_cast<const __nv_bfloat16*>(p.b);
  const __nv_bfloat16* q_ptr = static_cast<const __nv_bfloat16*>(p.q);
  const __nv_bfloat16* k_ptr = static_cast<const __nv_bfloat16*>(p.k);
  const __nv_bfloat16* v_ptr = static_cast<const __nv_bfloat16*>(p.v);
  const float A_log = p.A_log[h], dt_bias = p.dt_bias[h];
  // inputs of one token: raw gates, q, k (this lane's 16 elements), v of this
  // thread's rows
  struct Tok {
    float ga, gb, kf[16], qf[16], vv[U];
  };
  auto load_tok = [&](int t, Tok& x) {
    const int64_t bt = bidx * p.T + t;
    x.ga = __bfloat162float(a_ptr[bt * p.Hv + h]);
    x.gb = __bfloat162float(b_ptr[bt * p.Hv + h]);
    ld_vec16<BF16>(k_ptr + (bt * p.Hq + qh) * kHead, j, x.kf);
    ld_vec16<BF16>(q_ptr + (bt * p.Hq + qh) * kHead, j, x.qf);
#pragma unroll
    for (int u = 0; u < U; ++u) x.vv[u] = __bfloat162float(v_ptr[(bt * p.Hv + h) * kHead + row0 + 4 * u]);
  };
  Tok cur;
  load_tok(0, cur);
  for (int t = 0; t < p.T; ++t) {
    Tok nxt;
    if (MTP && t + 1 < p.T) load_tok(t + 1, nxt);
    const int64_t bt = bidx * p.T + t;
    const float g = expf(log_decay(A_log, cur.ga, dt_bias));
    const float beta = sigmoidf_acc(cur.gb);
    if constexpr (L2NORM) {
      float sk = 0.0f, sq = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        sk = fmaf(cur.kf[c], cur.kf[c], sk);
        sq = fmaf(cur.qf[c], cur.qf[c], sq);
      }
      const float rk = rsqrtf(octet_sum(sk) + 1e-6f), rq = rsqrtf(octet_sum(sq) + 1e-6f);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        cur.kf[c] *= rk;
        cur.qf[c] *= rq;
      }
    }
    __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (bt * p.Hv + h) * kHead;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int row = row0 + 4 * u;
      float dot = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        s[u][c] *= g;
        dot = fmaf(cur.kf[c], s[u][c], dot);
      }
      const float delta = beta * (cur.vv[u] - octet_sum(dot));
      float ov = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        s[u][c] = fmaf(cur.kf[c], delta, s[u][c]);
        ov = fmaf(cur.qf[c], s[u][c], ov);
      }
      ov = octet_sum(ov);
      if (j == 0) orow[row] = __float2bfloat16_rn(p.scale * ov);
      if (INTER && p.intermediate)
        store_row16<BF16>(p.intermediate, (bt * p.Hv + h) * kTile + static_cast<int64_t>(row) * kHead, j, s[u]);
    }
    if (MTP && t + 1 < p.T) cur = nxt;
  }

  if (write_back) {
    const int64_t base = (static_cast<int64_t>(sout) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead;
#pragma unroll
    for (int u = 0; u < U; ++u) store_row16<BF16>(p.pool, base + u * 4 * kHead, j, s[u]);
  }
}

// Single-token step on a bf16 pool: the loaded rows stay packed (two bf16 per
// register) until their turn, so a thread holds 8 rows -- as many bytes in flight
// as the fp32 form's 4 -- and each row is updated and written back right away.
// 128 threads (4 warps x 4 octets x 8 rows = one head's 128 rows), 4 CTAs per SM.
constexpr int kPackedThreads = 128, kPackedU = 8;

template <bool L2NORM>
__global__ void __launch_bounds__(kPackedThreads, 4) gdn_decode_pool_bf16_kernel(DecodePoolArgs p) {
  constexpr int U = kPackedU;
  const int64_t bh = blockIdx.x;  // b * Hv + h
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int oct = lane >> 3;
  const int j = lane & 7;
  const int row0 = warp * (4 * U) + oct;  // rows row0 + 4u
  constexpr int64_t kTile = kHead * kHead;

  const int32_t sin = p.in_slots[bidx];
  const int32_t sout = p.out_slots ? p.out_slots[bidx] : sin;
  const bool has_in = sin >= 0 && sin < p.pool_size;
  const bool write_back = !p.no_state_update && sout >= 0 && sout < p.pool_size;

  uint4 sp[U][2];  // this lane's 16 bf16 of each row (k = 64 i + 8 j + c)
  if (has_in) {
    const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(p.pool) +
                                (static_cast<int64_t>(sin) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead + 8 * j;
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int i = 0; i < 2; ++i) sp[u][i] = ld_stream_u4(base + u * 4 * kHead + 64 * i);
  } else {
#pragma unroll
    for (int u = 0; u < U; ++u) sp[u][0] = sp[u][1] = make_uint4(0u, 0u, 0u, 0u);
  }

  const int64_t bt = bidx;  // one token: bt = b
  const float g = expf(log_decay(p.A_log[h], __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[bt * p.Hv + h]),
                                 p.dt_bias[h]));
  const float beta = sigmoidf_acc(__bfloat162float(static_cast<const __nv_bfloat16*>(p.b)[bt * p.Hv + h]));
  float kf[16], qf[16];
  ld_vec16<true>(static_cast<const __nv_bfloat16*>(p.k) + (bt * p.Hq + qh) * kHead, j, kf);
  ld_vec16<true>(static_cast<const __nv_bfloat16*>(p.q) + (bt * p.Hq + qh) * kHead, j, qf);
  if constexpr (L2NORM) {
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
  const __nv_bfloat16* vrow = static_cast<const __nv_bfloat16*>(p.v) + (bt * p.Hv + h) * kHead;
  __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (bt * p.Hv + h) * kHead;
  __nv_bfloat16* wbase = static_cast<__nv_bfloat16*>(p.pool) +
                         (static_cast<int64_t>(sout) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead + 8 * j;
  __nv_bfloat16* ibase = p.intermediate ? static_cast<__nv_bfloat16*>(p.intermediate) + bh * kTile +
                                              static_cast<int64_t>(row0) * kHead + 8 * j
                                        : nullptr;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    float s[16];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t w[4] = {sp[u][i].x, sp[u][i].y, sp[u][i].z, sp[u][i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[8 * i + 2 * e] = bf16_lo(w[e]);
        s[8 * i + 2 * e + 1] = bf16_hi(w[e]);
      }
    }
    const int row = row0 + 4 * u;
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      s[c] *= g;
      dot = fmaf(kf[c], s[c], dot);
    }
    const float delta = beta * (__bfloat162float(vrow[row]) - octet_sum(dot));
    float ov = 0.0f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      s[c] = fmaf(kf[c], delta, s[c]);
      ov = fmaf(qf[c], s[c], ov);
    }
    ov = octet_sum(ov);
    if (j == 0) orow[row] = __float2bfloat16_rn(p.scale * ov);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 w = make_uint4(pack_bf16x2(s[8 * i + 0], s[8 * i + 1]), pack_bf16x2(s[8 * i + 2], s[8 * i + 3]),
                                 pack_bf16x2(s[8 * i + 4], s[8 * i + 5]), pack_bf16x2(s[8 * i + 6], s[8 * i + 7]));
      if (write_back) st_stream_u4(wbase + u * 4 * kHead + 64 * i, w);
      if (ibase) st_stream_u4(ibase + u * 4 * kHead + 64 * i, w);
    }
  }
}

// Multi-token steps on a bf16 pool, row by row: the T tokens' q, k (normalised
// here when asked), v and gates are staged in shared memory first, then each
// thread takes its 8 packed rows one at a time through all T tokens (fp32 between
// tokens, one bf16 rounding per store) -- the state stream keeps the bytes in flight
// of the single-token form instead of holding every row in fp32 across tokens.
// Shared memory per token: q, k, v as fp32 (3 x 512 B) + g, beta.  INTER: the
// per-token state cache is written (a separate instantiation: a runtime test per
// row and token costs the token loop ~11 %).
constexpr int kMtpMaxT = 32;

// Octet sums of four rows at once (lane j of the octet holds x[r], its share of
// row r's sum): a transposed butterfly -- at step 1 lanes j, j^1 swap two rows,
// at step 2 lanes j, j^2 one row, then a full exchange with j^4 -- leaves the sum
// of row 2 (j & 1) + ((j >> 1) & 1) in lanes j and j^4: 4 shuffles and 4 adds for
// the four rows instead of 12 and 12.
__device__ __forceinline__ float octet_sum4(const float (&x)[4], int j) {
  const bool b0 = j & 1, b1 = j & 2;
  const float s0 = b0 ? x[0] : x[2], s1 = b0 ? x[1] : x[3];
  const float k0 = b0 ? x[2] : x[0], k1 = b0 ? x[3] : x[1];
  const float y0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 1);
  const float y1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 1);
  const float z = (b1 ? y1 : y0) + __shfl_xor_sync(0xffffffffu, b1 ? y0 : y1, 2);
  return z + __shfl_xor_sync(0xffffffffu, z, 4);
}
// The octet lane that holds row r's sum after octet_sum4 (also lane + 4).
__device__ __forceinline__ int octet_sum4_lane(int r) { return (r >> 1) | ((r & 1) << 1); }

template <bool L2NORM, bool INTER>
__global__ void __launch_bounds__(kPackedThreads, 3) gdn_decode_pool_bf16_mtp_kernel(DecodePoolArgs p) {
  constexpr int U = kPackedU;
  extern __shared__ __align__(16) float tok[];  // [T][384]: q | k | v, then [T][2]: g, beta
  const int T = static_cast<int>(p.T);
  float* gb = tok + T * 3 * kHead;
  const int64_t bh = blockIdx.x;  // b * Hv + h
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int oct = lane >> 3;
  const int j = lane & 7;
  const int row0 = warp * (4 * U) + oct;
  constexpr int64_t kTile = kHead * kHead;

  const int32_t sin = p.in_slots[bidx];
  const int32_t sout = p.out_slots ? p.out_slots[bidx] : sin;
  const bool has_in = sin >= 0 && sin < p.pool_size;
  const bool write_back = !p.no_state_update && sout >= 0 && sout < p.pool_size;

  uint4 sp[U][2];
  if (has_in) {
    const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(p.pool) +
                                (static_cast<int64_t>(sin) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead + 8 * j;
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int i = 0; i < 2; ++i) sp[u][i] = ld_stream_u4(base + u * 4 * kHead + 64 * i);
  } else {
#pragma unroll
    for (int u = 0; u < U; ++u) sp[u][0] = sp[u][1] = make_uint4(0u, 0u, 0u, 0u);
  }

  // stage the tokens: warp w takes tokens w, w + 4, ...; lane l holds elements 4l..4l+3
  for (int t = warp; t < T; t += kPackedThreads / 32) {
    const int64_t bt = bidx * p.T + t;
    float qv[4], kv[4];
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.q) + (bt * p.Hq + qh) * kHead + 4 * lane, qv);
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.k) + (bt * p.Hq + qh) * kHead + 4 * lane, kv);
    if constexpr (L2NORM) {
      float sq = 0.0f, sk = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sq = fmaf(qv[c], qv[c], sq);
        sk = fmaf(kv[c], kv[c], sk);
      }
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, d);
        sk += __shfl_xor_sync(0xffffffffu, sk, d);
      }
      const float rq = rsqrtf(sq + 1e-6f), rk = rsqrtf(sk + 1e-6f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        qv[c] *= rq;
        kv[c] *= rk;
      }
    }
    float vv[4];
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.v) + (bt * p.Hv + h) * kHead + 4 * lane, vv);
    float* dst = tok + t * 3 * kHead + 4 * lane;
    *reinterpret_cast<float4*>(dst) = make_float4(qv[0], qv[1], qv[2], qv[3]);
    *reinterpret_cast<float4*>(dst + kHead) = make_float4(kv[0], kv[1], kv[2], kv[3]);
    *reinterpret_cast<float4*>(dst + 2 * kHead) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    if (lane == 0) {
      gb[2 * t] = expf(log_decay(p.A_log[h], __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[bt * p.Hv + h]),
                                 p.dt_bias[h]));
      gb[2 * t + 1] = sigmoidf_acc(__bfloat162float(static_cast<const __nv_bfloat16*>(p.b)[bt * p.Hv + h]));
    }
  }
  __syncthreads();

  __nv_bfloat16* wbase = static_cast<__nv_bfloat16*>(p.pool) +
                         (static_cast<int64_t>(sout) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead + 8 * j;
  // two rows at a time (independent chains), each token's dot products split in
  // two partial sums
  constexpr int R = 4;
#pragma unroll
  for (int u0 = 0; u0 < U; u0 += R) {
    float s[R][16];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t w[4] = {sp[u0 + r][i].x, sp[u0 + r][i].y, sp[u0 + r][i].z, sp[u0 + r][i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[r][8 * i + 2 * e] = bf16_lo(w[e]);
          s[r][8 * i + 2 * e + 1] = bf16_hi(w[e]);
        }
      }
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      const float* tq = tok + t * 3 * kHead;
      float kf[16], qf[16];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float4 k4 = *reinterpret_cast<const float4*>(tq + kHead + 64 * i + 8 * j + 4 * hh);
          const float4 q4 = *reinterpret_cast<const float4*>(tq + 64 * i + 8 * j + 4 * hh);
          kf[8 * i + 4 * hh + 0] = k4.x;
          kf[8 * i + 4 * hh + 1] = k4.y;
          kf[8 * i + 4 * hh + 2] = k4.z;
          kf[8 * i + 4 * hh + 3] = k4.w;
          qf[8 * i + 4 * hh + 0] = q4.x;
          qf[8 * i + 4 * hh + 1] = q4.y;
          qf[8 * i + 4 * hh + 2] = q4.z;
          qf[8 * i + 4 * hh + 3] = q4.w;
        }
      const float g = gb[2 * t], beta = gb[2 * t + 1];
      // element pairs (c, c + 1) on the packed FMUL2 / FFMA2 path: each lane
      // rounds like the scalar operation, and the pair's two lanes are the two
      // partial sums of every dot product
      float dot[R][2];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          const float2 sv = __fmul2_rn(make_float2(s[r][c], s[r][c + 1]), make_float2(g, g));
          s[r][c] = sv.x;
          s[r][c + 1] = sv.y;
          d2 = __ffma2_rn(make_float2(kf[c], kf[c + 1]), sv, d2);
        }
        dot[r][0] = d2.x;
        dot[r][1] = d2.y;
      }
      float delta[R];
      {
        static_assert(R == 4, "octet_sum4 reduces four rows");
        float part[4];
#pragma unroll
        for (int r = 0; r < R; ++r) part[r] = dot[r][0] + dot[r][1];
        const float red = octet_sum4(part, j);
        const int obase = lane & ~7;
#pragma unroll
        for (int r = 0; r < R; ++r)
          delta[r] = beta * (tq[2 * kHead + row0 + 4 * (u0 + r)] -
                             __shfl_sync(0xffffffffu, red, obase + octet_sum4_lane(r)));
      }
      float ov[R][2];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float2 o2 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          const float2 sv = __ffma2_rn(make_float2(kf[c], kf[c + 1]), make_float2(delta[r], delta[r]),
                                       make_float2(s[r][c], s[r][c + 1]));
          s[r][c] = sv.x;
          s[r][c + 1] = sv.y;
          o2 = __ffma2_rn(make_float2(qf[c], qf[c + 1]), sv, o2);
        }
        ov[r][0] = o2.x;
        ov[r][1] = o2.y;
      }
      const int64_t bt = bidx * p.T + t;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (bt * p.Hv + h) * kHead + row0 + 4 * u0;
      {
        float part[4];
#pragma unroll
        for (int r = 0; r < R; ++r) part[r] = ov[r][0] + ov[r][1];
        const float o = octet_sum4(part, j);  // row 2 (j & 1) + ((j >> 1) & 1)
        if (j < 4) orow[4 * (2 * (j & 1) + ((j >> 1) & 1))] = __float2bfloat16_rn(p.scale * o);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + 4 * (u0 + r);
        if (INTER) {
          __nv_bfloat16* ip = static_cast<__nv_bfloat16*>(p.intermediate) + (bt * p.Hv + h) * kTile +
                              static_cast<int64_t>(row) * kHead + 8 * j;
#pragma unroll
          for (int i = 0; i < 2; ++i)
            st_stream_u4(ip + 64 * i, make_uint4(pack_bf16x2(s[r][8 * i + 0], s[r][8 * i + 1]),
                                                 pack_bf16x2(s[r][8 * i + 2], s[r][8 * i + 3]),
                                                 pack_bf16x2(s[r][8 * i + 4], s[r][8 * i + 5]),
                                                 pack_bf16x2(s[r][8 * i + 6], s[r][8 * i + 7])));
        }
      }
    }
    if (write_back) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int i = 0; i < 2; ++i)
          st_stream_u4(wbase + (u0 + r) * 4 * kHead + 64 * i,
                       make_uint4(pack_bf16x2(s[r][8 * i + 0], s[r][8 * i + 1]),
                                  pack_bf16x2(s[r][8 * i + 2], s[r][8 * i + 3]),
                                  pack_bf16x2(s[r][8 * i + 4], s[r][8 * i + 5]),
                                  pack_bf16x2(s[r][8 * i + 6], s[r][8 * i + 7])));
    }
  }
}

// Multi-token step on an fp32 pool, the same scheme as the bf16 one above: the
// tokens staged in shared memory once per CTA, a thread's rows held in registers
// across all of them, the four rows' dot products reduced together (octet_sum4)
// and element pairs on the packed FMUL2 / FFMA2 path.  fp32 rows take twice the
// registers, so a CTA of 128 threads owns 64 rows (two CTAs per head, four rows
// per thread, all 16 loads of a thread issued at once) and four CTAs share an SM.
constexpr int kF32MtpRows = 64;

template <bool L2NORM, bool INTER>
__global__ void __launch_bounds__(kPackedThreads, 4) gdn_decode_pool_f32_mtp_kernel(DecodePoolArgs p) {
  constexpr int R = 4;  // rows per thread
  extern __shared__ __align__(16) float tok[];  // [T][384]: q | k | v, then [T][2]: g, beta
  const int T = static_cast<int>(p.T);
  float* gb = tok + T * 3 * kHead;
  const int64_t bh = blockIdx.x >> 1;  // b * Hv + h
  const int half = static_cast<int>(blockIdx.x & 1);
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int oct = lane >> 3;
  const int j = lane & 7;
  const int row0 = half * kF32MtpRows + warp * (4 * R) + oct;  // rows row0 + 4 r
  constexpr int64_t kTile = kHead * kHead;

  const int32_t sin = p.in_slots[bidx];
  const int32_t sout = p.out_slots ? p.out_slots[bidx] : sin;
  const bool has_in = sin >= 0 && sin < p.pool_size;
  const bool write_back = !p.no_state_update && sout >= 0 && sout < p.pool_size;

  float s[R][16];
  if (has_in) {
    const int64_t base = (static_cast<int64_t>(sin) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead;
#pragma unroll
    for (int r = 0; r < R; ++r) load_row16<false>(p.pool, base + r * 4 * kHead, j, s[r]);
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < 16; ++c) s[r][c] = 0.0f;
  }

  // stage the tokens: warp w takes tokens w, w + 4, ...; lane l holds elements 4l..4l+3
  for (int t = warp; t < T; t += kPackedThreads / 32) {
    const int64_t bt = bidx * p.T + t;
    float qv[4], kv[4];
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.q) + (bt * p.Hq + qh) * kHead + 4 * lane, qv);
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.k) + (bt * p.Hq + qh) * kHead + 4 * lane, kv);
    if constexpr (L2NORM) {
      float sq = 0.0f, sk = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sq = fmaf(qv[c], qv[c], sq);
        sk = fmaf(kv[c], kv[c], sk);
      }
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, d);
        sk += __shfl_xor_sync(0xffffffffu, sk, d);
      }
      const float rq = rsqrtf(sq + 1e-6f), rk = rsqrtf(sk + 1e-6f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        qv[c] *= rq;
        kv[c] *= rk;
      }
    }
    float vv[4];
    ld_bf16x4(static_cast<const __nv_bfloat16*>(p.v) + (bt * p.Hv + h) * kHead + 4 * lane, vv);
    float* dst = tok + t * 3 * kHead + 4 * lane;
    *reinterpret_cast<float4*>(dst) = make_float4(qv[0], qv[1], qv[2], qv[3]);
    *reinterpret_cast<float4*>(dst + kHead) = make_float4(kv[0], kv[1], kv[2], kv[3]);
    *reinterpret_cast<float4*>(dst + 2 * kHead) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    if (lane == 0) {
      gb[2 * t] = expf(log_decay(p.A_log[h], __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[bt * p.Hv + h]),
                                 p.dt_bias[h]));
      gb[2 * t + 1] = sigmoidf_acc(__bfloat162float(static_cast<const __nv_bfloat16*>(p.b)[bt * p.Hv + h]));
    }
  }
  __syncthreads();

#pragma unroll 1
  for (int t = 0; t < T; ++t) {
    const float* tq = tok + t * 3 * kHead;
    // this lane's 16 elements of k and q: element 4 i + c is k[32 i + 4 j + c]
    float kf[16], qf[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 k4 = *reinterpret_cast<const float4*>(tq + kHead + 32 * i + 4 * j);
      const float4 q4 = *reinterpret_cast<const float4*>(tq + 32 * i + 4 * j);
      kf[4 * i + 0] = k4.x;
      kf[4 * i + 1] = k4.y;
      kf[4 * i + 2] = k4.z;
      kf[4 * i + 3] = k4.w;
      qf[4 * i + 0] = q4.x;
      qf[4 * i + 1] = q4.y;
      qf[4 * i + 2] = q4.z;
      qf[4 * i + 3] = q4.w;
    }
    const float g = gb[2 * t], beta = gb[2 * t + 1];
    float part[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        const float2 sv = __fmul2_rn(make_float2(s[r][c], s[r][c + 1]), make_float2(g, g));
        s[r][c] = sv.x;
        s[r][c + 1] = sv.y;
        d2 = __ffma2_rn(make_float2(kf[c], kf[c + 1]), sv, d2);
      }
      part[r] = d2.x + d2.y;
    }
    float delta[R];
    {
      const float red = octet_sum4(part, j);
      const int obase = lane & ~7;
#pragma unroll
      for (int r = 0; r < R; ++r)
        delta[r] = beta * (tq[2 * kHead + row0 + 4 * r] -
                           __shfl_sync(0xffffffffu, red, obase + octet_sum4_lane(r)));
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float2 o2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        const float2 sv = __ffma2_rn(make_float2(kf[c], kf[c + 1]), make_float2(delta[r], delta[r]),
                                     make_float2(s[r][c], s[r][c + 1]));
        s[r][c] = sv.x;
        s[r][c + 1] = sv.y;
        o2 = __ffma2_rn(make_float2(qf[c], qf[c + 1]), sv, o2);
      }
      part[r] = o2.x + o2.y;
    }
    const int64_t bt = bidx * p.T + t;
    __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + (bt * p.Hv + h) * kHead + row0;
    {
      const float o = octet_sum4(part, j);  // row 2 (j & 1) + ((j >> 1) & 1)
      if (j < 4) orow[4 * (2 * (j & 1) + ((j >> 1) & 1))] = __float2bfloat16_rn(p.scale * o);
    }
    if (INTER) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        store_row16<false>(p.intermediate,
                           (bt * p.Hv + h) * kTile + static_cast<int64_t>(row0 + 4 * r) * kHead, j, s[r]);
    }
  }
  if (write_back) {
    const int64_t base = (static_cast<int64_t>(sout) * p.Hv + h) * kTile + static_cast<int64_t>(row0) * kHead;
#pragma unroll
    for (int r = 0; r < R; ++r) store_row16<false>(p.pool, base + r * 4 * kHead, j, s[r]);
  }
}

template <int U, bool BF16>
cudaError_t launch_u(const DecodePoolArgs& a, cudaStream_t s) {
  const int64_t ctas = a.B * a.Hv * (kHead / (32 * U));
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>(ctas);
  if (a.T > 1) {
    if (a.qk_l2norm && a.intermediate)
      gdn_decode_pool_kernel<U, BF16, true, true><<<grid, kThreads, 0, s>>>(a);
    else if (a.qk_l2norm)
      gdn_decode_pool_kernel<U, BF16, true, true, false><<<grid, kThreads, 0, s>>>(a);
    else if (a.intermediate)
      gdn_decode_pool_kernel<U, BF16, false, true><<<grid, kThreads, 0, s>>>(a);
    else
      gdn_decode_pool_kernel<U, BF16, false, true, false><<<grid, kThreads, 0, s>>>(a);
  } else {
    if (a.qk_l2norm)
      gdn_decode_pool_kernel<U, BF16, true, false><<<grid, kThreads, 0, s>>>(a);
    else
      gdn_decode_pool_kernel<U, BF16, false, false><<<grid, kThreads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

template <bool BF16>
cudaError_t launch_dtype(const DecodePoolArgs& a, cudaStream_t s) {
  if (BF16 && a.T > 1 && a.T <= kMtpMaxT) {  // packed rows, tokens staged in shared memory
    const int64_t ctas = a.B * a.Hv;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(a.T) * (3 * kHead + 2) * sizeof(float);
    auto kernel = a.intermediate ? (a.qk_l2norm ? gdn_decode_pool_bf16_mtp_kernel<true, true>
                                                : gdn_decode_pool_bf16_mtp_kernel<false, true>)
                                 : (a.qk_l2norm ? gdn_decode_pool_bf16_mtp_kernel<true, false>
                                                : gdn_decode_pool_bf16_mtp_kernel<false, false>);
    // T > 11 stages more than the 48 KiB default (T = 32: 49,408 B)
    const cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kernel<<<static_cast<unsigned>(ctas), kPackedThreads, smem, s>>>(a);
    return cudaGetLastError();
  }
  if (!BF16 && a.T > 1 && a.T <= kMtpMaxT) {  // four fp32 rows per thread, tokens in shared memory
    const int64_t ctas = a.B * a.Hv * (kHead / kF32MtpRows);
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(a.T) * (3 * kHead + 2) * sizeof(float);
    auto kernel = a.intermediate ? (a.qk_l2norm ? gdn_decode_pool_f32_mtp_kernel<true, true>
                                                : gdn_decode_pool_f32_mtp_kernel<false, true>)
                                 : (a.qk_l2norm ? gdn_decode_pool_f32_mtp_kernel<true, false>
                                                : gdn_decode_pool_f32_mtp_kernel<false, false>);
    const cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kernel<<<static_cast<unsigned>(ctas), kPackedThreads, smem, s>>>(a);
    return cudaGetLastError();
  }
  const int64_t sms = device_sm_count();
  if (BF16 && a.T == 1 && a.B * a.Hv >= 2 * sms) {  // the packed single-token form
    const int64_t ctas = a.B * a.Hv;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (a.qk_l2norm)
      gdn_decode_pool_bf16_kernel<true><<<static_cast<unsigned>(ctas), kPackedThreads, 0, s>>>(a);
    else
      gdn_decode_pool_bf16_kernel<false><<<static_cast<unsigned>(ctas), kPackedThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  // enough CTAs to fill the SMs several times before the tile grows
  const int64_t tiles = a.B * a.Hv;
  // (multi-token: at most 64 rows per thread block, whose registers also hold
  // the next token's inputs)
  if (tiles >= 4 * sms && a.T == 1) return launch_u<4, BF16>(a, s);
  if (tiles >= 2 * sms) return launch_u<2, BF16>(a, s);
  return launch_u<1, BF16>(a, s);
}

}  // namespace

cudaError_t launch_decode_pool(const DecodePoolArgs& a, cudaStream_t s) {
  if (a.B == 0 || a.T == 0) return cudaSuccess;
  if (decode_pool_tc_supported(a)) return launch_decode_pool_tc(a, s);
  return a.state_bf16 ? launch_dtype<true>(a, s) : launch_dtype<false>(a, s);
}

}  // namespace gdn
