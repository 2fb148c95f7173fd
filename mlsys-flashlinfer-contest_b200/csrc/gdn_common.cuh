// Shared device helpers for the GDN kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

#ifndef GDN_CONSTANTS_DEFINED
#define GDN_CONSTANTS_DEFINED
constexpr int kHead = 128;   // head_size (K = V = 128, fixed by the definitions)
constexpr int kChunk = 64;   // chunk length of the chunked prefill
#endif

// ------------------------------------------------------------------ gates
// torch.nn.functional.softplus with beta=1, threshold=20 (the definitions call
// F.softplus(a + dt_bias)): identity above 20, log1p(exp(x)) below.
__device__ __forceinline__ float softplus_t20(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

// log of the multiplicative decay: log g = -exp(A_log) * softplus(a + dt_bias)
__device__ __forceinline__ float log_decay(float A_log, float a, float dt_bias) {
  return -expf(A_log) * softplus_t20(a + dt_bias);
}

__device__ __forceinline__ float sigmoidf_acc(float x) { return 1.0f / (1.0f + expf(-x)); }

// 2^x with the hardware approximation, subnormal results flushed to zero.  Used
// on decay factors exp(gamma_i - gamma_j) <= 1, where a flushed subnormal only
// drops a contribution already below 2^-126 of the kept terms.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softplus with torch's threshold (identity above 20) from the hardware
// ex2/lg2 approximations.  Below -15, log1p(e^x) equals e^x to fp32 precision,
// so that branch returns e^x directly instead of losing it in 1 + e^x.
__device__ __forceinline__ float softplus_t20_fast(float x) {
  if (x > 20.0f) return x;
  const float e = ex2_ftz(x * kLog2e);
  return x < -15.0f ? e : kLn2 * lg2_approx(1.0f + e);
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float sigmoid_fast(float x) {
  return rcp_approx(1.0f + ex2_ftz(-x * kLog2e));
}

// ------------------------------------------------------------------ bf16
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Pack two floats into bf16x2 (round to nearest even); `lo` lands in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ------------------------------------------------------------------ memory
// 128-bit streaming load (evict-first in L1 and L2): state tiles are read once.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.cs.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// 128-bit streaming store.
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// 4 consecutive bf16 (8 bytes) through the read-only path, widened to fp32.
__device__ __forceinline__ void ld_bf16x4(const __nv_bfloat16* p, float* out) {
  uint2 w;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(p));
  out[0] = bf16_lo(w.x);
  out[1] = bf16_hi(w.x);
  out[2] = bf16_lo(w.y);
  out[3] = bf16_hi(w.y);
}

// Sum over the 8 lanes of an aligned lane octet (lanes differing in bits 0..2).
__device__ __forceinline__ float octet_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

}  // namespace gdn
