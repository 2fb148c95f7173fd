// Segmented (sequence-parallel) prefill on top of the fused chunked kernel.
//
// The chunked kernel walks a (sequence, v-head) pair's chunks in order on one
// SM, so a call with few pairs leaves most of the 148 SMs idle (one long
// sequence of a few heads, or a head-sharded multi-GPU call).  The state update
// is affine in the state: over tokens a..b,
//     S_b = S_{a-1} P + F,   P = A_a ... A_b,  A_t = g_t (I - beta_t k_t k_t^T),
// F the final state of the same tokens from a zero state, and P the final state
// from the identity with v = 0 (rows of the "state" are then k rows).  So a
// sequence cut into G pieces at chunk boundaries runs as
//   pass 1 (one launch): piece 0 from the initial state (outputs written, its
//          final state = the start state of piece 1) and, for pieces 1..G-2,
//          F_g and P_g (outputs not written);
//   combine (one launch): S_{g+1} = S_g P_g + F_g for g = 1..G-2, fp32 on CUDA
//          cores;
//   pass 2 (one launch): pieces 1..G-1 from their start states (outputs, and the
//          final state of the last piece).
// The chain is about 2/G of the sequence's chunks long instead of all of them,
// for (3G-4)/G times the chunk work: worth it when the pairs fill few SMs.  The
// jobs are built on the device from cu_seqlens (a one-CTA kernel), so the host
// never reads the lengths.  The reference has no counterpart: its chunked
// pipeline (chunk_v12.py:36-116) runs one state scan per (sequence, head).
#include <mutex>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

// Scratch of the no-allocation entry (gdn_prefill_segmented_noalloc): the job
// tables and piece states of one segmented call, in a file-scope device array
// that every GPU loading this library holds until the process exits.  Host code
// must not pass the array's name to a kernel (on the host it is a stand-in, not
// a device address): its address on each device comes from cudaGetSymbolAddress.
// Every call writes each byte it reads before reading it, so nothing in it has to
// start at zero; calls that overlap on the GPU (two streams, two threads) share
// it and race.
static __device__ __align__(256) unsigned char g_segment_scratch[kNoAllocScratchBytes];

namespace {

constexpr size_t kStateBytes1 = static_cast<size_t>(kHead) * kHead * sizeof(float);

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct SegLayout {
  SegJob* jobs1;    // [N][2G-3]
  SegJob* jobs2;    // [N][G-1]
  int32_t* split;   // [N]: sequence cut into G pieces
  float* sin;       // [N][G-1][Hv][128][128]: start state of piece g (g = 1..G-1)
  float* fst;       // [N][G-2][Hv][128][128]: F_g (g = 1..G-2)
  float* pst;       // [N][G-2][Hv][128][128]: P_g
};

SegLayout carve(void* ws, int64_t N, int64_t Hv, int G, size_t* bytes) {
  SegLayout l{};
  uint8_t* base = static_cast<uint8_t*>(ws);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* p = base ? base + off : nullptr;
    off += align256(n);
    return p;
  };
  const size_t st = static_cast<size_t>(Hv) * kStateBytes1;
  const int64_t mid = G > 2 ? G - 2 : 0;
  l.jobs1 = reinterpret_cast<SegJob*>(take(static_cast<size_t>(N) * (2 * G - 3) * sizeof(SegJob)));
  l.jobs2 = reinterpret_cast<SegJob*>(take(static_cast<size_t>(N) * (G - 1) * sizeof(SegJob)));
  l.split = reinterpret_cast<int32_t*>(take(static_cast<size_t>(N) * sizeof(int32_t)));
  l.sin = reinterpret_cast<float*>(take(static_cast<size_t>(N) * (G - 1) * st));
  l.fst = reinterpret_cast<float*>(take(static_cast<size_t>(N) * mid * st));
  l.pst = reinterpret_cast<float*>(take(static_cast<size_t>(N) * mid * st));
  *bytes = off;
  return l;
}

// One thread per sequence: cut it into G pieces of equal chunk counts (when it
// has at least two chunks per piece) and write its jobs of both passes.
__global__ void gdn_segment_jobs_kernel(const int64_t* cu_seqlens, int64_t N, int64_t T, int64_t Hv,
                                        int G, const float* state, float* new_state, SegLayout l) {
  const int64_t st = Hv * kHead * kHead;  // floats of one sequence's (or piece's) states
  const int64_t mid = G > 2 ? G - 2 : 0;
  for (int64_t n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    const int64_t bos = min(max(cu_seqlens[n], int64_t(0)), T);
    const int64_t eos = min(max(cu_seqlens[n + 1], bos), T);
    const int64_t nch = (eos - bos + kChunk - 1) / kChunk;
    SegJob* j1 = l.jobs1 + n * (2 * G - 3);
    SegJob* j2 = l.jobs2 + n * (G - 1);
    const float* s0 = state ? state + n * st : nullptr;
    float* s_out = new_state + n * st;
    const SegJob none{0, 0, nullptr, nullptr, 0u, 0u};
    const bool split = nch >= 2 * G;
    l.split[n] = split ? 1 : 0;
    if (!split) {
      j1[0] = SegJob{bos, eos, s0, s_out, 0u, 0u};
      for (int j = 1; j < 2 * G - 3; ++j) j1[j] = none;
      for (int j = 0; j < G - 1; ++j) j2[j] = none;
      continue;
    }
    auto piece = [&](int g, int64_t* b, int64_t* e) {
      *b = bos + (g * nch / G) * kChunk;
      *e = min(bos + ((g + 1) * nch / G) * kChunk, eos);
    };
    auto sin = [&](int g) { return l.sin + ((n * (G - 1) + (g - 1)) * st); };
    int64_t b, e;
    piece(0, &b, &e);
    j1[0] = SegJob{b, e, s0, sin(1), 0u, 0u};
    for (int g = 1; g <= G - 2; ++g) {
      piece(g, &b, &e);
      float* f = l.fst + (n * mid + (g - 1)) * st;
      float* pm = l.pst + (n * mid + (g - 1)) * st;
      j1[2 * g - 1] = SegJob{b, e, nullptr, f, kJobNoOut, 0u};
      j1[2 * g] = SegJob{b, e, nullptr, pm, kJobIdentity | kJobNoV | kJobNoOut, 0u};
    }
    for (int g = 1; g <= G - 1; ++g) {
      piece(g, &b, &e);
      j2[g - 1] = SegJob{b, e, sin(g), g == G - 1 ? s_out : nullptr, 0u, 0u};
    }
  }
}

// S_{g+1} = S_g P_g + F_g for every cut sequence and head, g = 1..G-2.  Rows r of
// S_{g+1} depend only on rows r of S_g, so a CTA owns 8 rows of one head and
// walks g in order with its rows in shared memory (no CTA waits on another);
// small CTAs (4 warps, 20 KB of shared memory) let several share an SM.  A
// thread computes a 2 x 4 tile (rows 2w, 2w+1 of warp w; columns 4 lane .. +3):
// per k one float4 of P and two broadcast values of S for 8 FMAs.  P goes
// through shared memory 32 rows (16 KB) at a time, the next tile's loads in
// flight in registers while the current tile is used.
constexpr int kCombRows = 8;
constexpr int kCombThreads = 32 * kCombRows / 2;
constexpr int kCombKTile = 32;
constexpr int kCombTiles = kHead / kCombKTile;  // per g
__global__ void __launch_bounds__(kCombThreads) gdn_segment_combine_kernel(int64_t N, int64_t Hv, int G,
                                                                  SegLayout l) {
  const int64_t cta = blockIdx.x;
  const int rb = static_cast<int>(cta % (kHead / kCombRows));
  const int64_t nh = cta / (kHead / kCombRows);
  const int64_t n = nh / Hv, h = nh % Hv;
  if (n >= N || !l.split[n]) return;
  const int64_t hrow = h * kHead * kHead + rb * kCombRows * kHead;  // this CTA's rows of a state
  const int64_t hmat = h * kHead * kHead;
  const int64_t st = Hv * kHead * kHead;
  const int64_t mid = G - 2;
  __shared__ __align__(16) float s_s[kCombRows][kHead];
  __shared__ __align__(16) float p_s[kCombKTile][kHead];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int r0 = 2 * w, c0 = 4 * lane;
  {
    const float* S1 = l.sin + (n * (G - 1)) * st + hrow;  // piece 1's start state (from pass 1)
    for (int i = t; i < kCombRows * kHead / 4; i += kCombThreads)
      reinterpret_cast<float4*>(&s_s[0][0])[i] = reinterpret_cast<const float4*>(S1)[i];
  }
  // tile i of the whole walk: g = 1 + i / kCombTiles, rows 32 (i % kCombTiles) .. of P_g
  const int ntiles = (G - 2) * kCombTiles;
  auto tile_src = [&](int i) {
    const int g = 1 + i / kCombTiles;
    return reinterpret_cast<const float4*>(l.pst + (n * mid + (g - 1)) * st + hmat +
                                           (i % kCombTiles) * kCombKTile * kHead);
  };
  constexpr int kPer = kCombKTile * kHead / 4 / kCombThreads;  // float4 per thread and tile
  float4 nxt[kPer];  // this thread's share of the next tile
  {
    const float4* src = tile_src(0);
#pragma unroll
    for (int j = 0; j < kPer; ++j) nxt[j] = src[t + kCombThreads * j];
  }
  float acc[2][4];
  for (int i = 0; i < ntiles; ++i) {
    const int g = 1 + i / kCombTiles, k0 = (i % kCombTiles) * kCombKTile;
    if (k0 == 0) {  // a new g: start from F_g
      const float* F = l.fst + (n * mid + (g - 1)) * st + hrow;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float4 f = *reinterpret_cast<const float4*>(F + (r0 + r) * kHead + c0);
        acc[r][0] = f.x;
        acc[r][1] = f.y;
        acc[r][2] = f.z;
        acc[r][3] = f.w;
      }
    }
    __syncthreads();  // the previous tile is consumed (and s_s written)
#pragma unroll
    for (int j = 0; j < kPer; ++j) reinterpret_cast<float4*>(&p_s[0][0])[t + kCombThreads * j] = nxt[j];
    __syncthreads();
    if (i + 1 < ntiles) {
      const float4* src = tile_src(i + 1);
#pragma unroll
      for (int j = 0; j < kPer; ++j) nxt[j] = src[t + kCombThreads * j];
    }
#pragma unroll 8
    for (int k = 0; k < kCombKTile; ++k) {
      const float4 pk = *reinterpret_cast<const float4*>(&p_s[k][c0]);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float sv = s_s[r0 + r][k0 + k];
        acc[r][0] = fmaf(sv, pk.x, acc[r][0]);
        acc[r][1] = fmaf(sv, pk.y, acc[r][1]);
        acc[r][2] = fmaf(sv, pk.z, acc[r][2]);
        acc[r][3] = fmaf(sv, pk.w, acc[r][3]);
      }
    }
    if (k0 + kCombKTile == kHead) {  // S_{g+1} done: to the workspace and to s_s
      __syncthreads();  // every thread is done reading s_s for this g
      float* out = l.sin + (n * (G - 1) + g) * st + hrow;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float4 v = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        *reinterpret_cast<float4*>(out + (r0 + r) * kHead + c0) = v;
        *reinterpret_cast<float4*>(&s_s[r0 + r][c0]) = v;
      }
    }
  }
}

}  // namespace

size_t prefill_segments_bytes(int64_t N, int64_t Hv, int segments) {
  if (segments < 2 || N <= 0) return 0;
  size_t bytes = 0;
  carve(nullptr, N, Hv, segments, &bytes);
  return bytes;
}

cudaError_t launch_prefill_segmented(const PrefillArgs& a, int G, void* ws, size_t ws_bytes,
                                     cudaStream_t s) {
  if (G < 2 || a.N == 0 || a.T == 0) return launch_prefill_chunked(a, s);
  size_t need = 0;
  const SegLayout l = carve(ws, a.N, a.Hv, G, &need);
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return cudaErrorInvalidValue;
  const int64_t jt = 256;
  const int64_t jb = (a.N + jt - 1) / jt;
  gdn_segment_jobs_kernel<<<static_cast<unsigned>(jb > 1024 ? 1024 : jb), jt, 0, s>>>(
      a.cu_seqlens, a.N, a.T, a.Hv, G, a.state, a.new_state, l);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PrefillArgs p1 = a;
  p1.jobs = l.jobs1;
  p1.njobs = a.N * (2 * G - 3);
  if ((e = launch_prefill_chunked(p1, s)) != cudaSuccess) return e;
  if (G > 2) {
    const int64_t cctas = a.N * a.Hv * (kHead / kCombRows);
    if (cctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_segment_combine_kernel<<<static_cast<unsigned>(cctas), kCombThreads, 0, s>>>(a.N, a.Hv, G, l);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  PrefillArgs p2 = a;
  p2.jobs = l.jobs2;
  p2.njobs = a.N * (G - 1);
  return launch_prefill_chunked(p2, s);
}

// Device address of g_segment_scratch on the current device, looked up on the
// first call on that device (then cached).
cudaError_t launch_prefill_segmented_noalloc(const PrefillArgs& a, int segments, cudaStream_t s) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
      void* p = nullptr;
      if ((e = cudaGetSymbolAddress(&p, g_segment_scratch)) != cudaSuccess) return e;
      addr[dev] = p;
    }
    ptr = addr[dev];
  }
  return launch_prefill_segmented(a, segments, ptr, kNoAllocScratchBytes, s);
}

}  // namespace gdn
