// Segmented (sequence-parallel) prefill on top of the fused chunked kernel.
//
// The chunked kernel walks a (sequence, v-head) pair's chunks in order on one
// SM, so a call with few pairs leaves most of the 148 SMs idle (one long
// sequence of a few heads, or a head-sharded multi-GPU call).  The state update
// is affine in the state: over tokens a..b,
//     S_b = S_{a-1} P + F,   P = A_a ... A_b,  A_t = g_t (I - beta_t k_t k_t^T),
// F the final state of the same tokens from a zero state, and P the final state
// from the identity with v = 0 (rows of the "state" are then k rows).  So a
// sequence cut into p pieces at chunk boundaries runs as
//   pass 1 (one launch): piece 0 from the initial state (outputs written, its
//          final state = the start state of piece 1) and, for pieces 1..p-2,
//          F_g and P_g (outputs not written);
//   combine (one launch): S_{g+1} = S_g P_g + F_g for g = 1..p-2, fp32 on CUDA
//          cores, each S_{g+1} written over F_g;
//   pass 2 (one launch): pieces 1..p-1 from their start states (outputs, and the
//          final state of the last piece).
// Piece 0 may be w times as long as the others (w "shares" of the sequence out
// of w + p - 1): pass 1 then lasts w shares, and the 2 (p - 2) F/P jobs of every
// cut sequence may take w waves of the SMs that the piece-0 jobs leave free.
// The chain is (w + 1) shares of the sequence instead of all of it, for
// (w + 3 (p - 1) - 2) / (w + p - 1) times the chunk work: worth it when the pairs
// fill few SMs.  The jobs are built on the device from cu_seqlens (a one-CTA
// kernel), so the host never reads the lengths.  With an automatic count the
// host gives only an upper bound and the job builder picks w and each
// sequence's count from its length (a ragged batch cuts its long sequences
// more), for the shortest longest chain whose pass 1 fits w waves, whose pass 2
// fits one and whose piece states fit the pool, and drops the cut when it would
// not shorten the longest chain; a forced count cuts every sequence of at least
// 2G chunks into G equal pieces (w = 1).
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
                    // state of piece 1, then F_1..F_{p-2} (the combine overwrites
                    // F_g with the start state of piece g + 1), then P_1..P_{p-2}
  int64_t cap;      // states in the pool
};

// States a cut into p pieces keeps: the start state of piece 1 + p - 2 of F
// (later the start states of pieces 2..p-1) + p - 2 of P.
__host__ __device__ inline int64_t states_of(int p) { return p >= 2 ? 2 * p - 3 : 0; }

// Pool size: a forced count keeps N (2G - 3) states; an automatic one at most
// 1.5 sms / Hv (the job builder keeps every cut within it; a one-wave pass 1,
// sum of Hv (2p - 3) over cut sequences <= sms, always fits).
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

// Chunk-times of one combine step (S_{g+1} = S_g P_g + F_g runs p - 2 of them
// one after the other), charged to a cut's chain when its piece count is chosen,
// and the fixed cost of cutting at all: the job builder, the combine and the
// second pass launch one after the other, ~25 us before any piece work (their
// launches, the combine's first loads, two more first chunks), about six
// chunk-times.  Without it, short sequences were cut where the extra launches
// cost more than the shorter chain saved (5 x 606 tokens at 8 heads: 77 us cut
// against 52 us whole).
constexpr int kCombineChunks = 1;
constexpr int kCutChunks = 6;

// floor(a / b) and ceil(a / b) for 0 <= a < 2^26, 1 <= b: a float estimate
// (off by a few units at most) set right by integer checks; an integer division
// is a long dependent chain, and the builder's search runs hundreds of them
// back to back.  No product below exceeds a + b.
__device__ __forceinline__ int floor_div(int a, int b) {
  int q = __float2int_rz(__fdividef(static_cast<float>(a), static_cast<float>(b)));
  while (q > 0 && q * b > a) --q;
  while ((q + 1) * b <= a) ++q;
  return q;
}
__device__ __forceinline__ int ceil_div(int a, int b) { return floor_div(a + b - 1, b); }

// Pieces of a c-chunk sequence in a cut call whose time is to stay within x
// chunk-times (x below the longest sequence, so the call is cut): the call takes
// pass 1 + the fixed cost + the combine + pass 2, and with piece 0 of w shares of
// a sequence and every other piece one share, pass 1 lasts w times pass 2.  So a
// sequence stays whole (1) when it fits pass 1, c <= w floor((x - kCutChunks) /
// (w + 1)) (a longer whole sequence would hold pass 2 back); else it takes the
// fewest p in [3, g] (two pieces would run one after the other, no shorter than
// the whole) with pieces of at least 2 chunks and (w + 1) ceil(c / (w + p - 1)) +
// kCombineChunks (p - 2) <= x - kCutChunks; 0 when there is none.  No p below the
// one whose shares are at most (x - kCutChunks) / (w + 1) chunks can do, so the
// count starts there.
__device__ int pieces_for_chain(int c, int x, int g, int w) {
  const int xr = x - kCutChunks;  // what is left for the pieces and the combine
  if (xr < 2 * (w + 1)) return 0;
  const int q = floor_div(xr, w + 1);
  if (c <= w * q) return 1;
  // no count reaches a chain below 2 sqrt((w + 1) c) - w - 1 ((w + 1) c / S + S,
  // S = w + p - 1, is at least twice the root of the product): most candidates
  // of the search end here, without the walk below
  if (static_cast<float>(xr) < 2.0f * sqrtf(static_cast<float>((w + 1) * c)) - w - 2) return 0;
  for (int p = max(ceil_div(c, q) - w + 1, 3); p <= g; ++p) {
    const int shares = w + p - 1;
    if (c < 2 * shares) return 0;
    if ((w + 1) * ceil_div(c, shares) + kCombineChunks * (p - 2) <= xr) return p;
  }
  return 0;
}

// Three warps, one per w, search the automatic form side by side; warp 0 then
// places every sequence's states in the pool and all three write the jobs of
// both passes.
// Automatic form: for w = 1, 2, 3 the shortest
// call time x in chunk-times (search over 1..longest; x = longest is the uncut
// call) whose pieces (pieces_for_chain: whole sequences within pass 1, cut ones
// within pass 1 + the fixed cost + the combine + pass 2) have F/P jobs, 2 Hv (p -
// 2) per cut sequence, that fit w waves of the SMs that pass 1's N Hv piece-0 (or
// whole-sequence) jobs leave free, pass-2 jobs, Hv (p - 1) per cut sequence, that
// fit one wave, and states that fit the pool; the w with the shortest x wins
// (ties: the smaller w), and nothing is cut unless x is at most 4/5 of the
// longest sequence.  With w = 1 the first rule is the one-wave pass 1
// of equal pieces.  Job tables are job-major (slot j of every sequence, then
// slot j + 1), so a grid's piece-0 jobs come before its F/P jobs and its real
// jobs before its empty ones.
constexpr int kJobWarps = 3;  // one per w
__global__ void __launch_bounds__(32 * kJobWarps) gdn_segment_jobs_kernel(
    const int64_t* cu_seqlens, int64_t N, int64_t T, int64_t Hv, int G, int adaptive, int sms,
    const float* state, float* new_state, SegLayout l) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __shared__ int s_x[kJobWarps];
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
  int x = 0;  // automatic form: the accepted chain (0: no cut)
  int w = 1;  // shares of piece 0
  if (adaptive) {
    // chunk counts of this lane's sequences, held in registers for the search
    // (beyond 4 per lane they are read again); the host only sends calls of at
    // most SMs / 2 (sequence, head) pairs here, so every sum fits 32 bits
    constexpr int kCached = 4;
    int cc[kCached];
    unsigned m = 0;
#pragma unroll
    for (int i = 0; i < kCached; ++i) {
      const int64_t n = lane + 32 * i;
      cc[i] = n < N ? static_cast<int>(chunks(n)) : 0;
      m = max(m, static_cast<unsigned>(cc[i]));
    }
    for (int64_t n = lane + 32 * kCached; n < N; n += 32)
      m = max(m, static_cast<unsigned>(chunks(n)));
    const int cmax = static_cast<int>(__reduce_max_sync(0xffffffffu, m));
    const int64_t free_sms = static_cast<int64_t>(sms) - N * Hv;
    auto feasible = [&](int xx, int ww) {
      unsigned fp = 0, p2 = 0, sts = 0;
      bool bad = false;
      auto add = [&](int c) {
        const int p = pieces_for_chain(c, xx, G, ww);
        bad |= p == 0;
        if (p >= 3) {
          fp += static_cast<unsigned>(2 * Hv * (p - 2));
          p2 += static_cast<unsigned>(Hv * (p - 1));
          sts += static_cast<unsigned>(states_of(p));
        }
      };
#pragma unroll
      for (int i = 0; i < kCached; ++i)
        if (lane + 32 * i < N) add(cc[i]);
      for (int64_t n = lane + 32 * kCached; n < N; n += 32) add(static_cast<int>(chunks(n)));
      if (__any_sync(0xffffffffu, bad)) return false;
      return __reduce_add_sync(0xffffffffu, fp) <= ww * free_sms &&
             __reduce_add_sync(0xffffffffu, p2) <= static_cast<unsigned>(sms) &&
             __reduce_add_sync(0xffffffffu, sts) <= l.cap;
    };
    // this warp's w: the shortest feasible x in [1, cmax] (x = cmax: nothing is
    // cut, feasible without a test; below it feasibility only grows with x).  Up to 32 sequences, the
    // warp tests 32 / lpc candidates per round (lpc = N rounded up to a power of
    // two lanes each, a sequence per lane), narrowing [lo, hi] that much per
    // round; beyond that, a binary search whose tests sum over the lanes'
    // sequences.
    const int ww = wid + 1;
    int lo = 1, hi = cmax;
    if (free_sms <= 0) {
      lo = cmax;
    } else if (N <= 32) {
      // lanes in groups of lpc (the power of two >= N), one sequence per lane and
      // one candidate x per group: 32 / lpc candidates per round, the group's sums
      // by xor shuffles within it
      const int lpc = N <= 1 ? 1 : 1 << (32 - __clz(static_cast<int>(N) - 1));
      const int nc = 32 / lpc, ci = lane / lpc, si = lane % lpc;
      const int cs = si < N ? cc[0] : 0;  // chunks of this lane's sequence
      const int c_mine = __shfl_sync(0xffffffffu, cs, si);  // lane si holds sequence si
      while (lo < hi) {
        const int span = hi - lo;  // candidates in [lo, hi); hi is feasible
        const int xj = span <= nc ? lo + ci : lo + static_cast<int>((int64_t(span) * ci) / nc);
        const bool valid = xj < hi;
        unsigned fp = 0, p2 = 0, sts = 0;
        bool bad = false;
        if (valid && si < N) {
          const int pc = pieces_for_chain(c_mine, xj, G, ww);
          bad = pc == 0;
          if (pc >= 3) {
            fp = static_cast<unsigned>(2 * Hv * (pc - 2));
            p2 = static_cast<unsigned>(Hv * (pc - 1));
            sts = static_cast<unsigned>(states_of(pc));
          }
        }
        for (int o = 1; o < lpc; o <<= 1) {
          fp += __shfl_xor_sync(0xffffffffu, fp, o);
          p2 += __shfl_xor_sync(0xffffffffu, p2, o);
          sts += __shfl_xor_sync(0xffffffffu, sts, o);
          bad |= __shfl_xor_sync(0xffffffffu, static_cast<int>(bad), o) != 0;
        }
        const bool ok = valid && !bad && fp <= ww * free_sms && p2 <= static_cast<unsigned>(sms) &&
                        sts <= l.cap;
        const unsigned okm = __ballot_sync(0xffffffffu, ok && si == 0);
        if (okm) {
          const int jl = __ffs(okm) - 1;  // leader lane of the smallest feasible candidate
          const int xprev = jl == 0 ? lo - 1 : __shfl_sync(0xffffffffu, xj, jl - lpc);
          hi = __shfl_sync(0xffffffffu, xj, jl);
          lo = xprev + 1;
        } else {
          lo = __shfl_sync(0xffffffffu, xj, 32 - lpc) + 1;  // every candidate below hi failed
          if (span <= nc) lo = hi;
        }
      }
    } else {
      while (lo < hi) {
        const int mid = (lo + hi) / 2;
        if (feasible(mid, ww)) hi = mid; else lo = mid + 1;
      }
    }
    if (lane == 0) s_x[wid] = lo;
    __syncthreads();
    int best = cmax;
    for (int j = 0; j < kJobWarps; ++j)
      if (s_x[j] < best) {
        best = s_x[j];
        w = j + 1;
      }
    if (cmax > 0 && 5 * best <= 4 * cmax) x = best;
    else w = 1;
  }
  auto pieces_of = [&](int64_t n) {
    const int64_t c = chunks(n);
    if (adaptive) return x > 0 ? max(pieces_for_chain(static_cast<int>(c), x, G, w), 1) : 1;
    return c >= 2 * G ? G : 1;
  };
  // per block of 32 sequences: warp 0 finds the pieces and pool bases (an
  // exclusive scan of the states; a sequence whose states would pass the pool's
  // end stays whole) into shared memory, then all threads write the block's job
  // table entries, one entry each, slot by slot
  __shared__ int s_p[32];
  __shared__ int64_t s_b0[32], s_bos[32], s_eos[32];
  const SegJob none{0, 0, nullptr, nullptr, 0u, 0u};
  const int s1 = 2 * G - 3, s2 = G - 1;  // slots per sequence in each pass
  int64_t running = 0;
  for (int64_t n0 = 0; n0 < N; n0 += 32) {
    const int nb = static_cast<int>(min(N - n0, int64_t(32)));
    if (wid == 0) {
      const int64_t n = n0 + lane;
      int p = n < N ? pieces_of(n) : 1;
      const int64_t need = states_of(p);
      int64_t incl = need;
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int64_t total = __shfl_sync(0xffffffffu, incl, 31);
      if (running + incl > l.cap) p = 1;
      if (n < N) {
        int64_t bos, eos;
        bounds(n, &bos, &eos);
        s_p[lane] = p;
        s_b0[lane] = running + incl - need;
        s_bos[lane] = bos;
        s_eos[lane] = eos;
        l.pieces[n] = p;
        l.base[n] = running + incl - need;
      }
      running += total;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < nb * (s1 + s2); idx += blockDim.x) {
      const int k = idx % nb, j = idx / nb;  // sequence n0 + k, slot j (pass 1, then pass 2)
      const int64_t n = n0 + k;
      const int p = s_p[k];
      const int64_t b0 = s_b0[k], bos = s_bos[k], eos = s_eos[k];
      const float* s0 = state ? state + n * st : nullptr;
      float* s_out = new_state + n * st;
      // share boundaries: piece 0 = shares [0, w), piece g >= 1 = share w + g - 1
      // (32-bit division: a sequence has at most 2^25 chunks and i <= 64 shares)
      const unsigned shares = static_cast<unsigned>(w + p - 1);
      const unsigned nch32 = static_cast<unsigned>((eos - bos + kChunk - 1) / kChunk);
      auto edge = [&](int i) {
        return min(bos + static_cast<int64_t>(static_cast<unsigned>(i) * nch32 / shares) * kChunk,
                   eos);
      };
      auto pb = [&](int g) { return g == 0 ? bos : edge(w + g - 1); };  // piece g: [pb(g), edge(w+g))
      auto pool = [&](int64_t i) { return l.pool + (b0 + i) * st; };
      // pool slots of a cut: 0 = start state of piece 1, 1..p-2 = F_g (then the
      // start state of piece g + 1), p-1..2p-4 = P_g
      SegJob jb = none;
      if (j < s1) {  // pass 1
        if (p < 2) {
          if (j == 0) jb = SegJob{bos, eos, s0, s_out, 0u, 0u};
        } else if (j == 0) {
          jb = SegJob{bos, edge(w), s0, pool(0), 0u, 0u};
        } else if (j <= 2 * p - 4) {
          const int g = (j + 1) / 2;
          jb = (j & 1) ? SegJob{pb(g), edge(w + g), nullptr, pool(g), kJobNoOut, 0u}
                       : SegJob{pb(g), edge(w + g), nullptr, pool(p - 1 + g - 1),
                                kJobIdentity | kJobNoV | kJobNoOut, 0u};
        }
        l.jobs1[j * N + n] = jb;
      } else {  // pass 2: piece g = j2 + 1 from its start state
        const int j2 = j - s1;
        if (p >= 2 && j2 < p - 1) {
          const int g = j2 + 1;
          jb = SegJob{pb(g), edge(w + g), pool(g - 1), g == p - 1 ? s_out : nullptr, 0u, 0u};
        }
        l.jobs2[j2 * N + n] = jb;
      }
    }
    __syncthreads();
  }
}

// S_{g+1} = S_g P_g + F_g for every cut sequence and head, g = 1..p-2, each
// written over F_g (the pool slot after S_g).  Rows r of S_{g+1} depend only on
// rows r of S_g and F_g, so a CTA owns 8 rows of one head and walks g in order
// with its rows in shared memory (no CTA waits on another, and a row of F_g is
// read before the same CTA overwrites it).  The 128-long sums are split over the
// CTA's 8 warps (16 k each), so a step is short even when few CTAs run: every
// lane holds an 8 x 4 tile (the CTA's rows, columns 4 lane .. +3), takes its 16
// rows of P_g straight from global memory (one float4 per k and lane: a warp
// reads 512 contiguous bytes) with all 16 loads in flight at once, the next
// step's issued as soon as this step's products are done, and the S values as
// broadcast float4 reads of four k of one row; the 8 partial tiles are summed
// through shared memory with F_g.  Every shared access is a float4 that is
// either broadcast or spread over all banks.
constexpr int kCombRows = 8;
constexpr int kCombWarps = 8;
constexpr int kCombThreads = 32 * kCombWarps;
constexpr int kCombK = kHead / kCombWarps;  // k per warp and step
__global__ void __launch_bounds__(kCombThreads, 2) gdn_segment_combine_kernel(int64_t N, int64_t Hv,
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
  float* sin = l.pool + b0 * st;                    // S_1, then F_g -> S_{g+1}
  const float* pst = l.pool + (b0 + (p - 1)) * st;  // P_1..P_{p-2}
  __shared__ __align__(16) float s_row[kCombRows][kHead];              // S_g rows
  __shared__ __align__(16) float red[kCombWarps][kCombRows][kHead];   // partial tiles
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int c0 = 4 * lane, k0 = w * kCombK;
  for (int i = t; i < kCombRows * kHead / 4; i += kCombThreads)  // S_1 (from pass 1)
    reinterpret_cast<float4*>(&s_row[0][0])[i] = reinterpret_cast<const float4*>(sin + hrow)[i];
  __syncthreads();
  auto load_p = [&](int g, float4* pk) {
    const float* P = pst + (g - 1) * st + hmat + static_cast<int64_t>(k0) * kHead + c0;
#pragma unroll
    for (int k = 0; k < kCombK; ++k) pk[k] = *reinterpret_cast<const float4*>(P + k * kHead);
  };
  float4 pk[kCombK];
  load_p(1, pk);
  const int rr = w;  // the row this thread sums
  for (int g = 1; g <= p - 2; ++g) {
    float* out = sin + g * st + hrow + rr * kHead + c0;  // F_g, then S_{g+1} over it
    float4 v = *reinterpret_cast<const float4*>(out);     // arrives during the products
    float acc[kCombRows][4];
#pragma unroll
    for (int r = 0; r < kCombRows; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.0f;
#pragma unroll
    for (int k4 = 0; k4 < kCombK; k4 += 4) {
#pragma unroll
      for (int r = 0; r < kCombRows; ++r) {
        const float4 sv = *reinterpret_cast<const float4*>(&s_row[r][k0 + k4]);
        const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          acc[r][0] = fmaf(s4[kk], pk[k4 + kk].x, acc[r][0]);
          acc[r][1] = fmaf(s4[kk], pk[k4 + kk].y, acc[r][1]);
          acc[r][2] = fmaf(s4[kk], pk[k4 + kk].z, acc[r][2]);
          acc[r][3] = fmaf(s4[kk], pk[k4 + kk].w, acc[r][3]);
        }
      }
    }
    if (g + 1 <= p - 2) load_p(g + 1, pk);
#pragma unroll
    for (int r = 0; r < kCombRows; ++r)
      *reinterpret_cast<float4*>(&red[w][r][c0]) =
          make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    __syncthreads();  // partial tiles written; every warp is done reading s_row
    // thread t sums column 4 (t % 32) .. +3 of row t / 32 over the warps, plus F_g
#pragma unroll
    for (int j = 0; j < kCombWarps; ++j) {
      const float4 q = *reinterpret_cast<const float4*>(&red[j][rr][c0]);
      v.x += q.x;
      v.y += q.y;
      v.z += q.z;
      v.w += q.w;
    }
    *reinterpret_cast<float4*>(out) = v;
    *reinterpret_cast<float4*>(&s_row[rr][c0]) = v;
    __syncthreads();  // S_{g+1} in s_row; red free
  }
}

}  // namespace

// The fewest chunks a sequence needs before the job builder's automatic form can
// accept any cut of it (x at most 4/5 of the sequence, pieces_for_chain's cost
// with the fixed cut cost); a call with fewer chunks in all cannot be cut.
int prefill_min_cut_chunks() {
  static const int c_min = [] {
    for (int c = 1; c < (1 << 16); ++c)
      for (int w = 1; w <= 3; ++w)
        for (int p = 3; 2 * (w + p - 1) <= c; ++p) {
          const int shares = w + p - 1;
          const int x = (w + 1) * ((c + shares - 1) / shares) + kCombineChunks * (p - 2) + kCutChunks;
          if (5 * x <= 4 * c) return c;
        }
    return 1 << 16;
  }();
  return c_min;
}

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
  gdn_segment_jobs_kernel<<<1, 32 * kJobWarps, 0, s>>>(a.cu_seqlens, a.N, a.T, a.Hv, G, adaptive ? 1 : 0, sms,
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
