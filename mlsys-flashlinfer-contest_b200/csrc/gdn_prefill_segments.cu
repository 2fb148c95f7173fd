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
// never reads the lengths.  With an automatic count the host gives only an upper
// bound and the job builder picks each sequence's count in proportion to its
// length (a ragged batch cuts its long sequences more), lowering the bound until
// pass 1 fits one wave of SMs and dropping the cut when it would not shorten the
// longest chain; a forced count cuts every sequence of at least 2G chunks into G.
// The reference has no counterpart: its chunked pipeline (chunk_v12.py:36-116)
// runs one state scan per (sequence, head).
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
  SegJob* jobs1;    // [2G-3][N] pass-1 jobs (G = the count or its upper bound)
  SegJob* jobs2;    // [G-1][N] pass-2 jobs
  int32_t* pieces;  // [N]: pieces of each sequence (1 = whole)
  int64_t* base;    // [N]: first state of each cut sequence in the pool
  float* pool;      // [cap][Hv][128][128]: per cut sequence with p pieces, the start
                    // states of pieces 1..p-1, then F_1..F_{p-2}, then P_1..P_{p-2}
  int64_t cap;      // states in the pool
};

// States a cut into p pieces keeps: p - 1 start states + 2 (p - 2) of F and P.
__host__ __device__ inline int64_t states_of(int p) { return p >= 2 ? 3 * p - 5 : 0; }

// Pool size: a forced count keeps N (3G - 5) states; an automatic one accepts a
// cut only when its pass 1, sum of Hv (2p - 3) over cut sequences, fits `sms`,
// and 3p - 5 <= 1.5 (2p - 3), so 1.5 sms / Hv states hold any accepted cut.
int64_t pool_states(int64_t N, int64_t Hv, int G, bool adaptive, int sms) {
  const int64_t full = N * states_of(G);
  if (!adaptive) return full;
  const int64_t bound = (3 * static_cast<int64_t>(sms)) / (2 * Hv);
  return full < bound ? full : bound;
}

SegLayout carve(void* ws, int64_t N, int64_t Hv, int G, bool adaptive, int sms, size_t* bytes) {
  SegLayout l{};
  uint8_t* base = static_cast<uint8_t*>(ws);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* p = base ? base + off : nullptr;
    off += align256(n);
    return p;
  };
  l.cap = pool_states(N, Hv, G, adaptive, sms);
  l.jobs1 = reinterpret_cast<SegJob*>(take(static_cast<size_t>(N) * (2 * G - 3) * sizeof(SegJob)));
  l.jobs2 = reinterpret_cast<SegJob*>(take(static_cast<size_t>(N) * (G - 1) * sizeof(SegJob)));
  l.pieces = reinterpret_cast<int32_t*>(take(static_cast<size_t>(N) * sizeof(int32_t)));
  l.base = reinterpret_cast<int64_t*>(take(static_cast<size_t>(N) * sizeof(int64_t)));
  l.pool = reinterpret_cast<float*>(take(static_cast<size_t>(l.cap) * Hv * kStateBytes1));
  *bytes = off;
  return l;
}

// Pieces of a c-chunk sequence that bring its chain (pass 1 + pass 2, 2 ceil(c /
// p) chunks; c when whole) down to x chunks: 1 when c <= x, else at least 3 (two
// pieces would run one after the other, no shorter than the whole), and 0 when
// no count within the bound g, with pieces of at least 2 chunks, does it.
__device__ int pieces_for_chain(int64_t c, int64_t x, int g) {
  if (c <= x) return 1;
  const int64_t half = x / 2;
  if (half < 1) return 0;
  const int64_t p = max((c + half - 1) / half, int64_t(3));
  return (p <= g && c >= 2 * p) ? static_cast<int>(p) : 0;
}

__device__ int64_t warp_sum(int64_t v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ int64_t warp_max(int64_t v) {
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp: choose every sequence's pieces, place their states in the pool and
// write the jobs of both passes.  Automatic form: the shortest chain x (binary
// search over 1..longest) whose pieces keep pass 1 within `sms` CTAs, sum of Hv
// (2p - 3) over cut sequences + Hv per whole one; no cut unless x is at most
// 4/5 of the longest sequence.  Job tables are job-major (slot j of every
// sequence, then slot j + 1), so a grid's real jobs come before its empty ones.
__global__ void __launch_bounds__(32) gdn_segment_jobs_kernel(
    const int64_t* cu_seqlens, int64_t N, int64_t T, int64_t Hv, int G, int adaptive, int sms,
    const float* state, float* new_state, SegLayout l) {
  const int lane = threadIdx.x;
  const int64_t st = Hv * kHead * kHead;  // floats of one sequence's (or piece's) states
  auto bounds = [&](int64_t n, int64_t* bos, int64_t* eos) {
    *bos = min(max(cu_seqlens[n], int64_t(0)), T);
    *eos = min(max(cu_seqlens[n + 1], *bos), T);
  };
  auto chunks = [&](int64_t n) {
    int64_t b, e;
    bounds(n, &b, &e);
    return (e - b + kChunk - 1) / kChunk;
  };
  int64_t x = 0;  // automatic form: the accepted chain (0: no cut)
  if (adaptive) {
    // chunk counts of this lane's sequences, held in registers for the search
    // (the host sends at most SMs / 3 sequences here; beyond 4 per lane they are
    // read again)
    constexpr int kCached = 4;
    int64_t cc[kCached];
    int64_t m = 0;
#pragma unroll
    for (int i = 0; i < kCached; ++i) {
      const int64_t n = lane + 32 * i;
      cc[i] = n < N ? chunks(n) : 0;
      m = max(m, cc[i]);
    }
    for (int64_t n = lane + 32 * kCached; n < N; n += 32) m = max(m, chunks(n));
    const int64_t cmax = warp_max(m);
    auto cost = [&](int64_t xx) {  // pass-1 CTAs for chain xx (huge when infeasible)
      int64_t cst = 0;
      auto add = [&](int64_t c) {
        const int p = pieces_for_chain(c, xx, G);
        cst += p == 0 ? (int64_t(1) << 40) : Hv * (p >= 3 ? 2 * p - 3 : 1);
      };
#pragma unroll
      for (int i = 0; i < kCached; ++i)
        if (lane + 32 * i < N) add(cc[i]);
      for (int64_t n = lane + 32 * kCached; n < N; n += 32) add(chunks(n));
      return warp_sum(cst);
    };
    int64_t lo = 1, hi = cmax;  // cost(cmax) = N Hv <= sms: feasible
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if (cost(mid) <= sms) hi = mid; else lo = mid + 1;
    }
    if (cmax > 0 && 5 * lo <= 4 * cmax) x = lo;
  }
  auto pieces_of = [&](int64_t n) {
    const int64_t c = chunks(n);
    if (adaptive) return x > 0 ? max(pieces_for_chain(c, x, G), 1) : 1;
    return c >= 2 * G ? G : 1;
  };
  // pieces and pool bases: an exclusive scan of the states over the sequences,
  // 32 at a time; a sequence whose states would pass the pool's end stays whole
  int64_t running = 0;
  for (int64_t n0 = 0; n0 < N; n0 += 32) {
    const int64_t n = n0 + lane;
    int p = n < N ? pieces_of(n) : 1;
    const int64_t need = states_of(p);
    int64_t incl = need;
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int64_t total = __shfl_sync(0xffffffffu, incl, 31);
    if (n < N) {
      if (running + incl > l.cap) p = 1;
      l.pieces[n] = p;
      l.base[n] = running + incl - need;
    }
    running += total;
  }
  // jobs (the same lane handled sequence n above)
  const SegJob none{0, 0, nullptr, nullptr, 0u, 0u};
  for (int64_t n = lane; n < N; n += 32) {
    int64_t bos, eos;
    bounds(n, &bos, &eos);
    const int64_t nch = (eos - bos + kChunk - 1) / kChunk;
    const int p = l.pieces[n];
    auto j1 = [&](int j) -> SegJob& { return l.jobs1[j * N + n]; };
    auto j2 = [&](int j) -> SegJob& { return l.jobs2[j * N + n]; };
    const float* s0 = state ? state + n * st : nullptr;
    float* s_out = new_state + n * st;
    for (int j = 0; j < 2 * G - 3; ++j) j1(j) = none;
    for (int j = 0; j < G - 1; ++j) j2(j) = none;
    if (p < 2) {
      j1(0) = SegJob{bos, eos, s0, s_out, 0u, 0u};
      continue;
    }
    const int64_t b0 = l.base[n];
    auto piece = [&](int g, int64_t* b, int64_t* e) {
      *b = bos + (g * nch / p) * kChunk;
      *e = min(bos + ((g + 1) * nch / p) * kChunk, eos);
    };
    auto sin = [&](int g) { return l.pool + (b0 + (g - 1)) * st; };
    auto fst = [&](int g) { return l.pool + (b0 + (p - 1) + (g - 1)) * st; };
    auto pst = [&](int g) { return l.pool + (b0 + (p - 1) + (p - 2) + (g - 1)) * st; };
    int64_t b, e;
    piece(0, &b, &e);
    j1(0) = SegJob{b, e, s0, sin(1), 0u, 0u};
    for (int g = 1; g <= p - 2; ++g) {
      piece(g, &b, &e);
      j1(2 * g - 1) = SegJob{b, e, nullptr, fst(g), kJobNoOut, 0u};
      j1(2 * g) = SegJob{b, e, nullptr, pst(g), kJobIdentity | kJobNoV | kJobNoOut, 0u};
    }
    for (int g = 1; g <= p - 1; ++g) {
      piece(g, &b, &e);
      j2(g - 1) = SegJob{b, e, sin(g), g == p - 1 ? s_out : nullptr, 0u, 0u};
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
__global__ void __launch_bounds__(kCombThreads) gdn_segment_combine_kernel(int64_t N, int64_t Hv,
                                                                           SegLayout l) {
  const int64_t cta = blockIdx.x;
  const int rb = static_cast<int>(cta % (kHead / kCombRows));
  const int64_t nh = cta / (kHead / kCombRows);
  const int64_t n = nh / Hv, h = nh % Hv;
  if (n >= N) return;
  const int p = l.pieces[n];
  if (p < 3) return;
  const int64_t hrow = h * kHead * kHead + rb * kCombRows * kHead;  // this CTA's rows of a state
  const int64_t hmat = h * kHead * kHead;
  const int64_t st = Hv * kHead * kHead;
  const int64_t b0 = l.base[n];
  const float* sin = l.pool + b0 * st;                    // start states of pieces 1..p-1
  const float* fst = l.pool + (b0 + (p - 1)) * st;        // F_1..F_{p-2}
  const float* pst = l.pool + (b0 + (2 * p - 3)) * st;    // P_1..P_{p-2}
  __shared__ __align__(16) float s_s[kCombRows][kHead];
  __shared__ __align__(16) float p_s[kCombKTile][kHead];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int r0 = 2 * w, c0 = 4 * lane;
  {
    const float* S1 = sin + hrow;  // piece 1's start state (from pass 1)
    for (int i = t; i < kCombRows * kHead / 4; i += kCombThreads)
      reinterpret_cast<float4*>(&s_s[0][0])[i] = reinterpret_cast<const float4*>(S1)[i];
  }
  // tile i of the whole walk: g = 1 + i / kCombTiles, rows 32 (i % kCombTiles) .. of P_g
  const int ntiles = (p - 2) * kCombTiles;
  auto tile_src = [&](int i) {
    const int g = 1 + i / kCombTiles;
    return reinterpret_cast<const float4*>(pst + (g - 1) * st + hmat +
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
      const float* F = fst + (g - 1) * st + hrow;
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
      float* out = const_cast<float*>(sin) + g * st + hrow;
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

size_t prefill_segments_bytes(int64_t N, int64_t Hv, int segments, bool adaptive, int sms) {
  if (segments < 2 || N <= 0) return 0;
  size_t bytes = 0;
  carve(nullptr, N, Hv, segments, adaptive, sms, &bytes);
  return bytes;
}

cudaError_t launch_prefill_segmented(const PrefillArgs& a, int G, bool adaptive, int sms, void* ws,
                                     size_t ws_bytes, cudaStream_t s) {
  if (G < 2 || a.N == 0 || a.T == 0) return launch_prefill_chunked(a, s);
  size_t need = 0;
  const SegLayout l = carve(ws, a.N, a.Hv, G, adaptive, sms, &need);
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return cudaErrorInvalidValue;
  gdn_segment_jobs_kernel<<<1, 32, 0, s>>>(a.cu_seqlens, a.N, a.T, a.Hv, G, adaptive ? 1 : 0, sms,
                                           a.state, a.new_state, l);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PrefillArgs p1 = a;
  p1.jobs = l.jobs1;
  p1.njobs = a.N * (2 * G - 3);
  if ((e = launch_prefill_chunked(p1, s)) != cudaSuccess) return e;
  if (G > 2) {
    const int64_t cctas = a.N * a.Hv * (kHead / kCombRows);
    if (cctas > 0x7fffffffLL) return cudaErrorInvalidValue;
    gdn_segment_combine_kernel<<<static_cast<unsigned>(cctas), kCombThreads, 0, s>>>(a.N, a.Hv, l);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  PrefillArgs p2 = a;
  p2.jobs = l.jobs2;
  p2.njobs = a.N * (G - 1);
  return launch_prefill_chunked(p2, s);
}

// Device address of g_segment_scratch on the current device, looked up on the
// first call on that device (then cached).
cudaError_t launch_prefill_segmented_noalloc(const PrefillArgs& a, int segments, bool adaptive,
                                             int sms, cudaStream_t s) {
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
  return launch_prefill_segmented(a, segments, adaptive, sms, ptr, kNoAllocScratchBytes, s);
}

}  // namespace gdn
