// Chunk metadata for the chunked prefill, computed on the device so the host
// never reads cu_seqlens (no device-to-host sync on the hot path).
//
// Same outputs as gdn_prefill/solution/python/cuda_prep_meta_v2.cu:11-70:
//   chunk_offsets[n] = number of 64-token chunks before sequence n (size N+1,
//                      chunk_offsets[N] = total);
//   chunk_indices[c] = (sequence, chunk-within-sequence) for every chunk c.
// The reference handles N <= 256 in one pass of <= 8 warps; here one CTA of 1024
// threads walks the sequences in blocks of 1024 with a running carry, so N is
// unbounded.  Entries of chunk_indices past the total are left untouched;
// writes that would pass max_chunks are dropped (the host sizes the array with
// the upper bound N + (T - N) / 64, so that only happens for inconsistent input).
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kMetaThreads = 1024;

__global__ void __launch_bounds__(kMetaThreads)
    gdn_prep_meta_kernel(const int64_t* __restrict__ cu, int64_t N, int32_t* __restrict__ offsets,
                         int32_t* __restrict__ indices, int64_t max_chunks) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry_s = 0;
    offsets[0] = 0;
  }
  __syncthreads();
  for (int64_t base = 0; base < N; base += kMetaThreads) {
    const int64_t n = base + tid;
    int32_t cnt = 0;
    if (n < N) {
      const int64_t len = cu[n + 1] - cu[n];
      cnt = len > 0 ? static_cast<int32_t>((len + kChunk - 1) / kChunk) : 0;
    }
    // inclusive scan within the warp
    int32_t x = cnt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_sums[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sums[lane] = w;  // inclusive prefix over warps
    }
    __syncthreads();
    const int32_t carry = carry_s;
    const int32_t incl = carry + x + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (n < N) {
      offsets[n + 1] = incl;
      const int32_t start = incl - cnt;
      for (int32_t c = 0; c < cnt; ++c) {
        if (start + c < max_chunks) {
          reinterpret_cast<int2*>(indices)[start + c] = make_int2(static_cast<int32_t>(n), c);
        }
      }
    }
    __syncthreads();
    if (tid == kMetaThreads - 1) carry_s = incl;
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_prep_meta(const int64_t* cu_seqlens, int64_t N, int32_t* chunk_offsets,
                             int32_t* chunk_indices, int64_t max_chunks, cudaStream_t s) {
  if (N < 0) return cudaErrorInvalidValue;
  gdn_prep_meta_kernel<<<1, kMetaThreads, 0, s>>>(cu_seqlens, N, chunk_offsets, chunk_indices,
                                                 max_chunks);
  return cudaGetLastError();
}

}  // namespace gdn
