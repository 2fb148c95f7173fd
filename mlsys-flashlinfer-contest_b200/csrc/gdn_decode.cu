// GDN decode: one fused pass over the fp32 recurrent state (sm_100a).
//
// Replaces gdn_decode/solution/python/gdn_decode_small_batch.cu:87-164 (B < 8)
// and gdn_decode/solution/python/gdn_decode_kernel_large_batch.py:18-254 (B >= 8)
// with one kernel for every batch size.
//
// Math per (sequence b, v-head h), state S[v][k] (k-last, fp32), following
// definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:91-132:
//   g = exp(-exp(A_log[h]) * softplus(a + dt_bias[h])),  beta = sigmoid(b)
//   old_v[v]  = sum_k k[k] * g * S[v][k]
//   S'[v][k]  = g * S[v][k] + k[k] * beta * (v[v] - old_v[v])
//   o[v]      = scale * sum_k q[k] * S'[v][k]
// Every state row v is independent, so the kernel is a pure stream: each row is
// read once, updated in registers and written once.
//
// Mapping: a CTA of 256 threads (8 warps) owns ROWS = 32*U consecutive rows of
// one (b, h) tile.  A warp owns 4*U rows; each aligned octet of 8 lanes owns one
// row at a time, a lane holding 16 of the row's 128 floats as four float4 at
// k = 32*i + 4*j (j = lane % 8), so every load instruction covers four fully used
// 128-byte segments.  All U rows of a lane are loaded before any is used (U*4
// independent 16-byte loads in flight per lane).  The two dot products reduce
// over the octet with three xor-shuffles each.
#include <stdlib.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kThreads = 256;

template <int U, bool HAS_STATE>
__global__ void __launch_bounds__(kThreads) gdn_decode_kernel(DecodeArgs p) {
  constexpr int kRows = 32 * U;
  constexpr int kTilesPerHead = kHead / kRows;
  const int64_t cta = blockIdx.x;
  const int64_t bh = cta / kTilesPerHead;           // b * Hv + h
  const int tile = static_cast<int>(cta % kTilesPerHead);
  const int64_t bidx = bh / p.Hv;
  const int h = static_cast<int>(bh % p.Hv);
  const int qh = h / static_cast<int>(p.Hv / p.Hq);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int oct = lane >> 3;
  const int j = lane & 7;
  const int row0 = tile * kRows + warp * (4 * U) + oct;  // rows row0 + 4u

  // State loads first: they are the long-latency part.
  float4 s[U][4];
  const int64_t tile_elem = bh * (kHead * kHead);
  if constexpr (HAS_STATE) {
    const float* sp = p.state + tile_elem + static_cast<int64_t>(row0) * kHead + 4 * j;
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[u][i] = ld_stream_f4(sp + u * 4 * kHead + 32 * i);
  }

  // Gates (per thread; a handful of transcendental ops).
  const __nv_bfloat16* a_ptr = static_cast<const __nv_bfloat16*>(p.a);
  const __nv_bfloat16* b_ptr = static_cast<const __nv_bfloat16*>(p.b);
  const float g = expf(log_decay(p.A_log[h], __bfloat162float(a_ptr[bh]), p.dt_bias[h]));
  const float beta = sigmoidf_acc(__bfloat162float(b_ptr[bh]));

  float kf[16], qf[16];
  {
    const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(p.k) + (bidx * p.Hq + qh) * kHead;
    const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(p.q) + (bidx * p.Hq + qh) * kHead;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ld_bf16x4(kp + 32 * i + 4 * j, kf + 4 * i);
      ld_bf16x4(qp + 32 * i + 4 * j, qf + 4 * i);
    }
  }
  const __nv_bfloat16* vrow = static_cast<const __nv_bfloat16*>(p.v) + bh * kHead;
  float vv[U];
#pragma unroll
  for (int u = 0; u < U; ++u) vv[u] = __bfloat162float(vrow[row0 + 4 * u]);

  float* np_ = p.new_state + tile_elem + static_cast<int64_t>(row0) * kHead + 4 * j;
  __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) + bh * kHead;

#pragma unroll
  for (int u = 0; u < U; ++u) {
    float old[16];
    if constexpr (HAS_STATE) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        old[4 * i + 0] = g * s[u][i].x;
        old[4 * i + 1] = g * s[u][i].y;
        old[4 * i + 2] = g * s[u][i].z;
        old[4 * i + 3] = g * s[u][i].w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 16; ++c) old[c] = 0.0f;
    }
    float dot = 0.0f;
    if constexpr (HAS_STATE) {
#pragma unroll
      for (int c = 0; c < 16; ++c) dot = fmaf(kf[c], old[c], dot);
      dot = octet_sum(dot);
    }
    const float delta = beta * (vv[u] - dot);
    float ov = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 w;
      w.x = fmaf(kf[4 * i + 0], delta, old[4 * i + 0]);
      w.y = fmaf(kf[4 * i + 1], delta, old[4 * i + 1]);
      w.z = fmaf(kf[4 * i + 2], delta, old[4 * i + 2]);
      w.w = fmaf(kf[4 * i + 3], delta, old[4 * i + 3]);
      st_stream_f4(np_ + u * 4 * kHead + 32 * i, w);
      ov = fmaf(qf[4 * i + 0], w.x, ov);
      ov = fmaf(qf[4 * i + 1], w.y, ov);
      ov = fmaf(qf[4 * i + 2], w.z, ov);
      ov = fmaf(qf[4 * i + 3], w.w, ov);
    }
    ov = octet_sum(ov);
    if (j == 0) op[row0 + 4 * u] = __float2bfloat16_rn(p.scale * ov);
  }
}

template <int U>
cudaError_t launch_u(const DecodeArgs& a, cudaStream_t s) {
  const int64_t ctas = a.B * a.Hv * (kHead / (32 * U));
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (a.state)
    gdn_decode_kernel<U, true><<<static_cast<unsigned>(ctas), kThreads, 0, s>>>(a);
  else
    gdn_decode_kernel<U, false><<<static_cast<unsigned>(ctas), kThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

// GDN_DECODE_ROWS_PER_CTA (32, 64 or 128) overrides the automatic tile choice;
// it is read once per process and exists for tuning sweeps.
static int rows_override() {
  static const int v = [] {
    const char* e = getenv("GDN_DECODE_ROWS_PER_CTA");
    const int r = e ? atoi(e) : 0;
    return (r == 32 || r == 64 || r == 128) ? r : 0;
  }();
  return v;
}

cudaError_t launch_decode(const DecodeArgs& a, int rows_per_cta, cudaStream_t s) {
  if (a.B == 0) return cudaSuccess;
  if (rows_per_cta == 0) rows_per_cta = rows_override();
  if (rows_per_cta == 0) {
    // Enough CTAs to fill the SMs several times over before growing the tile.
    const int64_t tiles = a.B * a.Hv, sms = device_sm_count();
    rows_per_cta = tiles >= 4 * sms ? 128 : (tiles >= 2 * sms ? 64 : 32);
  }
  switch (rows_per_cta) {
    case 32: return launch_u<1>(a, s);
    case 64: return launch_u<2>(a, s);
    case 128: return launch_u<4>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
