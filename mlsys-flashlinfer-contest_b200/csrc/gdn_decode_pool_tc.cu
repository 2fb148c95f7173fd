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
// triangular solve per row in fp32, and the rank-T update sum_tau w_tau k_tau as a
// second MMA whose A operand is the weights split into three bf16 terms (~24
// mantissa bits, an fp32 weight to rounding) and whose B operand is the bf16 k
// rows, accumulated in fp32.  The
// token-by-token form spends four multiply-adds per state element and token on CUDA
// cores; this one spends one per element for all T tokens.
//
// Persistent and warp-specialised: one CTA per SM walks (sequence, v-head) units
// blockIdx.x, blockIdx.x + gridDim.x, ... through an NS-stage shared-memory ring,
// each role a warp (or several) that hands off to the next through mbarriers:
//   * loader (warp 13): the unit's slots, then its state tile, k, q and v rows
//     and gate inputs by TMA (128-byte swizzle) as soon as a stage frees;
//   * issuer (warp 14): S_0 [K;Q]^T and the tokens' Gram [K;Q][K;Q]^T by tcgen05,
//     each into one of two TMEM buffers; update issuer (warp 16): the state update
//     MMA D2 = W K;
//   * gates (warp 15): decay g_t and beta_t of the unit's tokens;
//   * tables (warp 12, TMEM lanes 0-31): the Gram rows -> decay products and the
//     per-token factors of the solve and of the update;
//   * solve (warps 0-3, thread = state row): the row's 2T dot products from TMEM,
//     delta, the T outputs and the row's update weights w_tau delta_tau, written to
//     TMEM as three bf16 terms;
//   * update (warps 4-11): s_T = C s_0 + D2 into the state tile in shared memory,
//     stored to the pool by one TMA store, while the solve warps work on the next
//     unit.
// Every wait is bounded (2 s), after which the CTA sets a status bit and stops.
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

// Warp roles (TMEM lane quarter = warp % 4).
constexpr int kSolveWarps = 4;                  // warps 0-3: thread = state row (quarters 0-3)
constexpr int kUpdateWarps = 8;                 // warps 4-11: the new state, 16 rows each
constexpr int kTablesWarp = 12;                 // reads the Gram rows (lanes 0-31: quarter 0)
constexpr int kLoaderWarp = 13;                 // slots and TMA loads
constexpr int kIssuerWarp = 14;                 // tcgen05.mma issue
constexpr int kGatesWarp = 15;                  // decay and beta of every token
constexpr int kUpdIssuerWarp = 16;              // tcgen05.mma issue of the state update
constexpr int kThreads = 32 * 17;
constexpr uint32_t kUpdateBar = 1;  // named barrier of the update warps
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kStateBytes = kHead * kHead * 2;  // one bf16 state tile
constexpr uint32_t kKb = 16384;                      // one 64-column block of the state tile
constexpr int kMaxHv = 256;                          // A_log / dt_bias staged in shared memory

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t r;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(addr) : "memory");
  return r;
}

// A wait on the next step of the pipeline: polled closely first, then with
// short sleeps, bounded by kTimeoutNs.
__device__ __forceinline__ bool wait_step(uint64_t* bar, uint32_t parity) {
#pragma unroll 1
  for (int i = 0; i < 512; ++i)
    if (mbar_test(bar, parity)) return true;
  return mbar_wait_nap(bar, parity, kTimeoutNs);
}

constexpr uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// Shared-memory layout for a token-count bound TP (8 or 16); T <= TP.
template <int TP>
struct Lay {
  static constexpr int N1 = 2 * TP;            // token rows: k [0, TP), q [TP, 2 TP)
  static constexpr int NS = TP <= 8 ? 5 : 4;   // stages of the ring
  static constexpr uint32_t kTokKb = N1 * 128;  // one 64-column block of the token tile
  static constexpr uint32_t kVKb = TP * 128;    // one 64-column block of the v tile
  // one stage (offsets from its 1024-aligned base); the token tile comes first
  // so that the Gram MMA's 128-row A operand stays inside the stage
  static constexpr uint32_t ST_TOK = 0;                          // [kb 2][N1][128 B]
  static constexpr uint32_t ST_S = ST_TOK + 2 * kTokKb;          // [kb 2][128][128 B]
  static constexpr uint32_t ST_V = ST_S + kStateBytes;           // [kb 2][TP][128 B]
  static constexpr uint32_t ST_GA = ST_V + 2 * kVKb;             // a: [TP][8 heads] bf16
  static constexpr uint32_t ST_GB = ST_GA + align_up(TP * 16, 128);
  static constexpr uint32_t ST_TAB = ST_GB + align_up(TP * 16, 128);
  // tables: Ak[TP][TP], Bq[TP][TP], Ck[TP], Cq[TP], beta[TP], wgt[TP], the decay
  // products D[TP][TP], C[TP], D[T-1][t] (DW[TP]), C_final, out slot
  static constexpr int T_AK = 0, T_BQ = TP * TP, T_CK = 2 * TP * TP, T_CQ = T_CK + TP, T_BET = T_CQ + TP,
                       T_WGT = T_BET + TP, T_D = T_WGT + TP, T_C = T_D + TP * TP, T_DW = T_C + TP,
                       T_CF = T_DW + TP, T_SLOT = T_CF + 1;
  static constexpr uint32_t kTabFloats = T_SLOT + 3;
  static constexpr uint32_t kStage = align_up(ST_TAB + kTabFloats * 4, 1024);
  // CTA-wide: A_log and dt_bias, barriers
  static constexpr uint32_t OFF_HP = NS * kStage;
  static constexpr uint32_t OFF_BAR = OFF_HP + 2 * kMaxHv * 4;
  // per stage: full, gates, tables, empty; per TMEM buffer: S_0 [K;Q]^T done, read;
  // Gram done, read; update weights written; update MMA done; update read
  static constexpr int kBars = 4 * NS + 14;
  static constexpr uint32_t kBytes = OFF_BAR + kBars * 8 + 16 + 1024;
  // TMEM columns, two buffers of each: D1 (S_0 [K;Q]^T, N1), Gram (N1), the update
  // weights as three bf16 A operands (hi, mid, lo: 8 columns each), D2 (the update,
  // 128)
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t C_D1 = 0, C_G = 2 * N1, C_A2 = 4 * N1, C_D2 = 256;
  static_assert(C_A2 + 48 <= C_D2, "TMEM columns overlap");
};

template <int TP, bool L2NORM>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_decode_pool_tc_kernel(const __grid_constant__ CUtensorMap tm_pool,
                              const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v,
                              const __grid_constant__ CUtensorMap tm_a,
                              const __grid_constant__ CUtensorMap tm_b, DecodePoolArgs p) {
  using L = Lay<TP>;
  constexpr int NS = L::NS, N1 = L::N1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;            // TMA of stage s landed
  uint64_t* gater = bars + NS;      // gates of stage s written (gates warp)
  uint64_t* tabr = bars + 2 * NS;   // tables of stage s written (tables warp)
  uint64_t* empty = bars + 3 * NS;  // stage s consumed (update warps)
  uint64_t* mmab = bars + 4 * NS;   // S_0 [K;Q]^T in D1 buffer b (tcgen05.commit)
  uint64_t* freeb = mmab + 2;       // D1 buffer b read (solve warps)
  uint64_t* gramb = freeb + 2;      // Gram MMA of buffer b done
  uint64_t* gfree = gramb + 2;      // Gram buffer b read (tables warp)
  uint64_t* a2ready = gfree + 2;    // update weights of buffer b in TMEM (solve warps)
  uint64_t* d2full = a2ready + 2;   // the update MMA of buffer b done (tcgen05.commit)
  uint64_t* d2free = d2full + 2;    // D2 buffer b read (update warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBars);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  volatile int* waited_units = reinterpret_cast<volatile int*>(tmem_slot + 2);
  float* hA = reinterpret_cast<float*>(smem + L::OFF_HP);
  float* hD = hA + kMaxHv;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = static_cast<int>(p.T);
  const int64_t units = p.B * p.Hv;
  const int nh = blockIdx.x < units ? static_cast<int>((units - 1 - blockIdx.x) / gridDim.x) + 1 : 0;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&gater[i], 1);
      mbar_init(&tabr[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&mmab[i], 1);
      mbar_init(&freeb[i], kSolveWarps);
      mbar_init(&gramb[i], 1);
      mbar_init(&gfree[i], 1);
      mbar_init(&a2ready[i], kSolveWarps);
      mbar_init(&d2full[i], 1);
      mbar_init(&d2free[i], kUpdateWarps);
    }
    fence_mbar_init();
    *abort_flag = 0u;
    *waited_units = 0;
  }
  for (int i = tid; i < p.Hv; i += kThreads) {  // A_log and dt_bias of every head
    hA[i] = p.A_log[i];
    hD[i] = p.dt_bias[i];
  }
  // The token tiles start as zeros: TMA writes only rows [0, T) and [TP, TP + T),
  // and the update MMA multiplies rows [T, TP) by zero weights, which must not
  // meet a NaN bit pattern left in shared memory.
  for (int st = 0; st < NS; ++st)
    for (uint32_t i = tid; i < 2 * L::kTokKb / 16; i += kThreads)
      sts128(sb + st * L::kStage + L::ST_TOK + 16 * i, 0u, 0u, 0u, 0u);
  fence_async_smem();
  if (warp == kLoaderWarp && lane == 0) {
    prefetch_tmap(&tm_pool);
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;
  int issued = 0;  // loader: units whose loads were issued
  const auto unit_head = [&](int j) {
    return static_cast<int>((blockIdx.x + static_cast<int64_t>(j) * gridDim.x) % p.Hv);
  };
  const auto stage_tab = [&](int s) { return reinterpret_cast<float*>(smem + s * L::kStage + L::ST_TAB); };

  if (warp == kLoaderWarp) {
    // ============================ loader =====================================
    int slot_in = -1, slot_out = -1;  // slots of units 32 i + lane (this lane's share)
    for (int j = 0; j < nh; ++j) {
      const int s = j % NS;
      if ((j & 31) == 0) {  // slots of the next 32 units, one per lane
        const int jl = j + lane;
        if (jl < nh) {
          const int64_t bl = (blockIdx.x + static_cast<int64_t>(jl) * gridDim.x) / p.Hv;
          slot_in = p.in_slots[bl];
          slot_out = p.out_slots ? p.out_slots[bl] : slot_in;
        }
      }
      const int sin = __shfl_sync(0xffffffffu, slot_in, j & 31);
      const int sout = __shfl_sync(0xffffffffu, slot_out, j & 31);
      const int64_t bi = (blockIdx.x + static_cast<int64_t>(j) * gridDim.x) / p.Hv;
      const int h = unit_head(j);
      const int qh = h / static_cast<int>(p.Hv / p.Hq);
      const bool has_in = sin >= 0 && sin < p.pool_size;
      if (*abort_flag || (j >= NS && !mbar_wait_nap(&empty[s], ((j / NS) - 1) & 1, kTimeoutNs))) {
        failed = true;
        break;
      }
      uint8_t* st = smem + s * L::kStage;
      const uint32_t sst = sb + s * L::kStage;
      if (!has_in) {  // zero initial state: an all-zero tile
        for (uint32_t i = lane; i < kStateBytes / 16; i += 32) sts128(sst + L::ST_S + 16 * i, 0u, 0u, 0u, 0u);
        fence_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        reinterpret_cast<int*>(stage_tab(s))[L::T_SLOT] = sout;
        mbar_arrive_expect_tx(&full[s], (has_in ? kStateBytes : 0u) + 6u * T * 128u + 2u * T * 16u);
        if (has_in) {
          const int tile = static_cast<int>(static_cast<int64_t>(sin) * p.Hv + h);
          tma_load_3d(st + L::ST_S, &tm_pool, &full[s], 0, 0, tile);
          tma_load_3d(st + L::ST_S + kKb, &tm_pool, &full[s], 64, 0, tile);
        }
        const int tok = static_cast<int>(bi * p.T);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_3d(st + L::ST_TOK + kb * L::kTokKb, &tm_k, &full[s], kb * 64, qh, tok);
          tma_load_3d(st + L::ST_TOK + kb * L::kTokKb + TP * 128, &tm_q, &full[s], kb * 64, qh, tok);
          tma_load_3d(st + L::ST_V + kb * L::kVKb, &tm_v, &full[s], kb * 64, h, tok);
        }
        tma_load_2d(st + L::ST_GA, &tm_a, &full[s], h & ~7, tok);
        tma_load_2d(st + L::ST_GB, &tm_b, &full[s], h & ~7, tok);
      }
      issued = j + 1;
      __syncwarp();
    }
  } else if (warp == kIssuerWarp) {
    // ============================ MMA issuer =================================
    // Unit jj: S_0 [K;Q]^T and the Gram MMA once its loads landed.
    for (int jj = 0; jj < nh; ++jj) {
      const int s = jj % NS, b = jj & 1;
      const uint32_t sst = sb + s * L::kStage;
      if (*abort_flag || !wait_step(&full[s], (jj / NS) & 1) ||
          (jj >= 2 && (!wait_step(&freeb[b], ((jj >> 1) - 1) & 1) ||
                       !wait_step(&gfree[b], ((jj >> 1) - 1) & 1)))) {
        failed = true;
        break;
      }
      if (lane == 0) *waited_units = jj + 1;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t tok16 = (sst + L::ST_TOK) >> 4, s16 = (sst + L::ST_S) >> 4;
        const uint32_t idesc = idesc_bf16(128, N1, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // S_0 [K;Q]^T -> D1 buffer b
          const uint64_t a = sdesc_sw128_f(s16 + ((ks >> 2) * kKb + (ks & 3) * 32) / 16, 16, 1024);
          const uint64_t bd = sdesc_sw128_f(tok16 + ((ks >> 2) * L::kTokKb + (ks & 3) * 32) / 16, 16, 1024);
          mma_bf16_ss(tmem + L::C_D1 + b * N1, a, bd, idesc, ks > 0);
        }
        mma_commit(&mmab[b]);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {  // [K;Q][K;Q]^T -> Gram buffer b (rows >= N1 unused)
          const uint64_t d = sdesc_sw128_f(tok16 + ((ks >> 2) * L::kTokKb + (ks & 3) * 32) / 16, 16, 1024);
          mma_bf16_ss(tmem + L::C_G + b * N1, d, d, idesc, ks > 0);
        }
        mma_commit(&gramb[b]);
      }
      __syncwarp();
    }
  } else if (warp == kUpdIssuerWarp) {
    // ============================ update MMA issuer ==========================
    // Unit u: D2 = W_hi K + W_mid K + W_lo K (W: the solve warps' update weights
    // split into three bf16 terms in TMEM, ~24 mantissa bits in all; K: the token
    // tile read as an MN-major operand), once the weights are in TMEM and the
    // update warps have read D2 buffer b for unit u - 2.
    for (int u = 0; u < nh; ++u) {
      const int s = u % NS, b = u & 1;
      if (*abort_flag || !wait_step(&a2ready[b], (u >> 1) & 1) ||
          (u >= 2 && !wait_step(&d2free[b], ((u >> 1) - 1) & 1))) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t tok16 = (sb + s * L::kStage + L::ST_TOK) >> 4;
        const uint64_t bk = sdesc_sw128_f(tok16, L::kTokKb, 1024);
        const uint32_t idesc = idesc_bf16(128, 128, false, true);
#pragma unroll
        for (int part = 0; part < 3; ++part)
          mma_bf16_ts(tmem + L::C_D2 + 128 * b, tmem + L::C_A2 + 24 * b + 8 * part, bk, idesc, part > 0);
        mma_commit(&d2full[b]);
      }
      __syncwarp();
    }
  } else if (warp == kGatesWarp) {
    // ============================ gates ======================================
    for (int jj = 0; jj < nh; ++jj) {
      const int s = jj % NS;
      const uint32_t sst = sb + s * L::kStage;
      if (*abort_flag || !wait_step(&full[s], (jj / NS) & 1)) {
        failed = true;
        break;
      }
      const int h = unit_head(jj);
      float* tab = stage_tab(s);
      // token `lane`: its rows of 8 heads hold this head at h & 7; lanes >= T carry
      // g = 1 through the products below
      float gl = 1.f;
      if (lane < T) {
        const float a = __uint_as_float(lds_u16(sst + L::ST_GA + lane * 16 + (h & 7) * 2) << 16);
        const float bb = __uint_as_float(lds_u16(sst + L::ST_GB + lane * 16 + (h & 7) * 2) << 16);
        gl = expf(log_decay(hA[h], a, hD[h]));
        tab[L::T_BET + lane] = sigmoidf_acc(bb);
      }
      // C_t = g_0 ... g_t (inclusive product scan) and the suffix products
      // g_t ... g_{T-1}; D[T-1][t] = the suffix product from t + 1
      float c = gl, suf = gl;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, c, d);
        const float z = __shfl_down_sync(0xffffffffu, suf, d);
        if (lane >= d) c *= y;
        if (lane + d < 32) suf *= z;
      }
      const float dw = __shfl_down_sync(0xffffffffu, suf, 1);
      // row t of D: D[t][tau] = g_{tau+1} ... g_t for tau <= t
      float dd = 1.f;
#pragma unroll
      for (int tau = TP - 1; tau >= 0; --tau) {
        const float gt = __shfl_sync(0xffffffffu, gl, tau);
        if (lane < TP && tau <= lane) {
          tab[L::T_D + lane * TP + tau] = dd;
          dd *= gt;
        }
      }
      if (lane < TP) {
        tab[L::T_C + lane] = c;
        tab[L::T_DW + lane] = lane + 1 < T ? dw : 1.f;
      }
      if (lane == T - 1) tab[L::T_CF] = c;
      __syncwarp();
      if (lane == 0) mbar_arrive(&gater[s]);
    }
  } else if (warp == kTablesWarp) {
    // ============================ tables =====================================
    for (int kk = 0; kk < nh; ++kk) {
      const int s = kk % NS, b = kk & 1;
      if (*abort_flag || !wait_step(&gater[s], (kk / NS) & 1) || !wait_step(&gramb[b], (kk >> 1) & 1)) {
        failed = true;
        break;
      }
      float* tab = stage_tab(s);
      // Gram products: lane m holds row m of [K;Q][K;Q]^T (k rows m < TP, q rows
      // TP + t), i.e. k_m . k_tau in column tau and q_t . k_tau on lane TP + t
      tc_fence_after();
      float g[N1];
#pragma unroll
      for (int c0 = 0; c0 < N1; c0 += 16) tmem_ld16(tmem + L::C_G + b * N1 + c0, g + c0);
      tmem_wait_ld();
      reg_fence(g);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&gfree[b]);
      // 1 / |k_tau| for every tau (lane tau holds k_tau . k_tau in column tau), and
      // 1 / |q_t| on lane TP + t (column TP + t)
      float rk[TP];
#pragma unroll
      for (int tau = 0; tau < TP; ++tau) {
        const float kk2 = __shfl_sync(0xffffffffu, g[tau], tau);
        rk[tau] = L2NORM ? rsqrtf(kk2 + 1e-6f) : 1.f;
      }
      // lane t < T: row t of Ak and Ck, wgt; lane TP + t: row t of Bq and Cq.  One
      // code path: the row factor, the diagonal mask and the target differ.
      const bool krow = lane < T, qrow = lane >= TP && lane < TP + T;
      const int t = krow ? lane : lane - TP;
      float rkt = 1.f, rq = 1.f;
#pragma unroll
      for (int i = 0; i < N1; ++i) {
        if (i < TP && i == t) rkt = rk[i];
        if (L2NORM && i == lane) rq = rsqrtf(g[i] + 1e-6f);
      }
      if (krow || qrow) {
        const float f = krow ? rkt : p.scale * rq;
        float* dst = tab + (krow ? L::T_AK : L::T_BQ) + t * TP;
        const float* drow = tab + L::T_D + t * TP;
#pragma unroll
        for (int tau = 0; tau < TP; ++tau) {
          const bool in = krow ? tau < t : tau <= t;
          if (tau <= t) dst[tau] = in ? f * drow[tau] * rk[tau] * g[tau] : 0.f;
        }
        const float ct = tab[L::T_C + t];
        if (krow) {
          tab[L::T_CK + t] = ct * rkt;
          tab[L::T_WGT + t] = tab[L::T_DW + t] * rkt;
        } else {
          tab[L::T_CQ + t] = f * ct;
        }
      } else if (lane >= T && lane < TP) {  // padding entries of the update weights
        tab[L::T_WGT + lane] = 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tabr[s]);
    }
  } else if (warp < kSolveWarps) {
    // ============================ solve (thread = state row) =================
    for (int jj = 0; jj < nh; ++jj) {
      const int s = jj % NS, b = jj & 1;
      const uint32_t sst = sb + s * L::kStage;
      if (*abort_flag || !wait_step(&tabr[s], (jj / NS) & 1) || !wait_step(&mmab[b], (jj >> 1) & 1)) {
        failed = true;
        break;
      }
      mbar_wait(&full[s], (jj / NS) & 1, kTimeoutNs);  // completed: acquires the stage's tiles
      const float* tab = stage_tab(s);
      const int64_t bi = (blockIdx.x + static_cast<int64_t>(jj) * gridDim.x) / p.Hv;
      const int h = unit_head(jj);
      tc_fence_after();
      float dk[N1];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + L::C_D1 + b * N1;
#pragma unroll
      for (int c0 = 0; c0 < N1; c0 += 16) tmem_ld16(taddr + c0, dk + c0);
      tmem_wait_ld();
      reg_fence(dk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&freeb[b]);
      // v[t][row] from the swizzled v tile
      const int row = tid, vkb = row >> 6, vcol = row & 63;
      const uint32_t vbase = sst + L::ST_V + vkb * L::kVKb + (vcol & 7) * 2;
      float delta[TP];
      __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) + (bi * p.T * p.Hv + h) * kHead + row;
#pragma unroll
      for (int t = 0; t < TP; ++t) {
        if (t < T) {
          const float vt = __uint_as_float(lds_u16(vbase + t * 128 + (((vcol >> 3) ^ (t & 7)) << 4)) << 16);
          float dt = tab[L::T_CK + t] * dk[t];
          float o = tab[L::T_CQ + t] * dk[TP + t];
#pragma unroll
          for (int tau = 0; tau < t; ++tau) {
            dt = fmaf(tab[L::T_AK + t * TP + tau], delta[tau], dt);
            o = fmaf(tab[L::T_BQ + t * TP + tau], delta[tau], o);
          }
          delta[t] = tab[L::T_BET + t] * (vt - dt);
          o = fmaf(tab[L::T_BQ + t * TP + t], delta[t], o);
          op[static_cast<int64_t>(t) * p.Hv * kHead] = __float2bfloat16_rn(o);
        } else {
          delta[t] = 0.f;
        }
      }
      // update weights w_tau delta_tau of this row as three bf16 A operands of the
      // update MMA, w = hi + mid + lo (K = 16 per operand; weights beyond T are
      // zero), once the update MMA of unit jj - 2 has read the buffer
      if (jj >= 2 && !wait_step(&d2full[b], ((jj >> 1) - 1) & 1)) {
        failed = true;
        break;
      }
      uint32_t whi[8], wmid[8], wlo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float w0 = 0.f, w1 = 0.f;
        if (2 * e < TP) w0 = tab[L::T_WGT + 2 * e] * delta[2 * e];
        if (2 * e + 1 < TP) w1 = tab[L::T_WGT + 2 * e + 1] * delta[2 * e + 1];
        whi[e] = pack_bf16x2(w0, w1);
        const float r0 = w0 - bf16_lo(whi[e]), r1 = w1 - bf16_hi(whi[e]);
        wmid[e] = pack_bf16x2(r0, r1);
        wlo[e] = pack_bf16x2(r0 - bf16_lo(wmid[e]), r1 - bf16_hi(wmid[e]));
      }
      const uint32_t a2 = tmem + (static_cast<uint32_t>(warp * 32) << 16) + L::C_A2 + 24 * b;
      tmem_st8u(a2, whi);
      tmem_st8u(a2 + 8, wmid);
      tmem_st8u(a2 + 16, wlo);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a2ready[b]);
    }
  } else if (warp < kSolveWarps + kUpdateWarps) {
    // ============================ update =====================================
    // s_T = C_{T-1} s_0 + D2: warp w reads TMEM lanes of quarter w % 4 (thread =
    // state row) and one 64-column half of D2; s_0 comes from the state tile in
    // shared memory, and s_T goes back into it, in place, for one TMA store of the
    // whole tile.
    const int quarter = warp & 3, half = (warp - kSolveWarps) >> 2;
    const int row = 32 * quarter + lane;
    const bool leader = warp == kSolveWarps && lane == 0;
    int prev_stage = -1;  // leader: stage whose store is still in flight
    for (int jj = 0; jj < nh; ++jj) {
      const int s = jj % NS, b = jj & 1;
      uint8_t* st = smem + s * L::kStage;
      const uint32_t sst = sb + s * L::kStage;
      if (*abort_flag || !wait_step(&d2full[b], (jj >> 1) & 1)) {
        failed = true;
        break;
      }
      mbar_wait(&full[s], (jj / NS) & 1, kTimeoutNs);  // completed: acquires the stage's tiles
      const float* tab = stage_tab(s);
      const float cfin = tab[L::T_CF];
      const int sout = reinterpret_cast<const int*>(tab)[L::T_SLOT];
      const bool store = !p.no_state_update && sout >= 0 && sout < p.pool_size;
      tc_fence_after();
      float d2[64];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + L::C_D2 + 128 * b + 64 * half;
      tmem_ld32(taddr, d2);
      tmem_ld32(taddr + 32, d2 + 32);
      tmem_wait_ld();
      reg_fence(d2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d2free[b]);
      if (store) {
        const uint32_t sblk = sst + L::ST_S + half * kKb;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunk c of this row's half
          const uint32_t addr = sblk + sw128_off(row, c);
          const uint4 s4 = lds128(addr);
          const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 v2 = __ffma2_rn(make_float2(bf16_lo(sw[e]), bf16_hi(sw[e])), make_float2(cfin, cfin),
                                         make_float2(d2[8 * c + 2 * e], d2[8 * c + 2 * e + 1]));
            o[e] = pack_bf16x2(v2.x, v2.y);
          }
          sts128(addr, o[0], o[1], o[2], o[3]);
        }
        fence_async_smem();
      }
      named_sync(kUpdateBar, 32 * kUpdateWarps);
      // One store group per unit (empty without write-back); a stage is released
      // once its tile has been read out, one unit later, so the leader never waits
      // for the store it just issued.
      if (leader) {
        if (store) {
          const int tile = static_cast<int>(static_cast<int64_t>(sout) * p.Hv + unit_head(jj));
          tma_store_3d(&tm_pool, st + L::ST_S, 0, 0, tile);
          tma_store_3d(&tm_pool, st + L::ST_S + kKb, 64, 0, tile);
        }
        bulk_commit();
        bulk_wait_read_1();
        if (prev_stage >= 0) mbar_arrive(&empty[prev_stage]);
        prev_stage = s;
      }
    }
    if (leader) {
      bulk_wait_all();
      if (prev_stage >= 0) mbar_arrive(&empty[prev_stage]);
    }
  }
  if (failed) {
    *abort_flag = 1u;
    atomicOr(&g_pool_tc_status, kStatusPoolTimeout);
  }
  __syncthreads();
  // loads still in flight (possible only after a timeout) land before the CTA exits
  if (warp == kLoaderWarp && lane == 0 && *abort_flag)
    for (int jx = *waited_units; jx < issued; ++jx) mbar_wait(&full[jx % NS], (jx / NS) & 1, kTimeoutNs);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

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

// [d2][d1][128] bf16 viewed with box {64, b1, b2}, 128-byte swizzle: the pool as
// [P*Hv tiles][128 rows][128] (box = one 64-column block of a tile) and q/k/v as
// [B*T][heads][128] (box = T token rows of one head, 64 columns).
cudaError_t encode_rows(CUtensorMap* m, const void* base, uint64_t d1, uint64_t d2, uint32_t b1,
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

// gate inputs [B*T][Hv] bf16, box = T rows of 8 heads (16 bytes), no swizzle
cudaError_t encode_gates(CUtensorMap* m, const void* base, uint64_t Hv, uint64_t rows, uint32_t T) {
  auto fn = encoder();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {Hv, rows};
  cuuint64_t strides[1] = {Hv * 2};
  cuuint32_t box[2] = {8, T};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int TP>
cudaError_t launch_tp(const DecodePoolArgs& a, cudaStream_t s) {
  using Lx = Lay<TP>;
  CUtensorMap mp, mq, mk, mv, ma, mb;
  cudaError_t e;
  const uint64_t rows = static_cast<uint64_t>(a.B * a.T);
  const uint32_t T = static_cast<uint32_t>(a.T);
  if ((e = encode_rows(&mp, a.pool, kHead, static_cast<uint64_t>(a.pool_size * a.Hv), 128, 1)) != cudaSuccess ||
      (e = encode_rows(&mq, a.q, a.Hq, rows, 1, T)) != cudaSuccess ||
      (e = encode_rows(&mk, a.k, a.Hq, rows, 1, T)) != cudaSuccess ||
      (e = encode_rows(&mv, a.v, a.Hv, rows, 1, T)) != cudaSuccess ||
      (e = encode_gates(&ma, a.a, a.Hv, rows, T)) != cudaSuccess ||
      (e = encode_gates(&mb, a.b, a.Hv, rows, T)) != cudaSuccess)
    return e;
  auto kernel = a.qk_l2norm ? gdn_decode_pool_tc_kernel<TP, true> : gdn_decode_pool_tc_kernel<TP, false>;
  if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), Lx::kBytes)) != cudaSuccess) return e;
  const int64_t units = a.B * a.Hv;
  const int64_t grid = units < device_sm_count() ? units : device_sm_count();
  kernel<<<static_cast<unsigned>(grid), kThreads, Lx::kBytes, s>>>(mp, mq, mk, mv, ma, mb, a);
  return cudaGetLastError();
}

}  // namespace

bool decode_pool_tc_supported(const DecodePoolArgs& a) {
  // bf16 pool, 3..16 tokens, no per-token state cache.  Measured on B200 at B = 256
  // and 64, Hv = 32 (us per step at B = 256, token-by-token kernel vs this one):
  // T = 2 107 vs 123, T = 3 127 vs 125, T = 4 150 vs 130, T = 8 259 vs 151,
  // T = 16 477 vs 258.  This kernel's cost per (sequence, head) is mostly fixed
  // (the per-unit hand-offs of its pipeline), the token-by-token kernel's grows with
  // T.  TMA needs 16-byte aligned bases and row strides (the gate rows, Hv bf16
  // values: Hv % 8 == 0).
  const auto al = [](const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; };
  return a.state_bf16 && a.T >= 3 && a.T <= 16 && a.intermediate == nullptr && a.pool_size > 0 &&
         a.Hv % 8 == 0 && a.Hv <= kMaxHv && al(a.pool) && al(a.q) && al(a.k) && al(a.v) && al(a.a) &&
         al(a.b) && a.pool_size * a.Hv <= 0x7fffffffLL && a.B * a.T <= 0x7fffffffLL;
}

cudaError_t read_pool_tc_status(uint32_t* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_pool_tc_status, sizeof(uint32_t));
  if (e != cudaSuccess || !clear) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_pool_tc_status, &zero, sizeof(uint32_t));
}

cudaError_t launch_decode_pool_tc(const DecodePoolArgs& a, cudaStream_t s) {
  if (a.B == 0) return cudaSuccess;
  return a.T <= 8 ? launch_tp<8>(a, s) : launch_tp<16>(a, s);
}

}  // namespace gdn
