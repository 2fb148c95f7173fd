// GDN prefill, chunked (C = 64) WY/UT form on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's 4-kernel pipeline chunk_v12.py:36-116
// (prep_meta_v2 -> kkt_inv_uw_v1 -> h_v2b -> o_v1) with ONE fused kernel: a
// CTA owns one (sequence, v-head) and walks its chunks in order, keeping the
// fp32 state in TMEM for the whole sequence.  Nothing is materialised in HBM
// between the stages (the reference writes U/W, per-chunk bf16 state
// snapshots h and v_new, i.e. ~2 KiB/token/head of extra traffic).
//
// Per chunk (tokens t, s in [0,64), gamma = within-chunk cumulative log decay,
// S = [K,V] state at the chunk start, St = S^T = k-last [V,K] in TMEM):
//   G|QK  = [K;Q] K^T                          (tcgen05, M=128: rows 0-63 KK^T, 64-127 QK^T)
//   A     = strict_tril(beta_t G e^{gamma_t - gamma_s}),  P = tril(QK e^{gamma_t - gamma_s})
//   T     = (I + A)^-1                         (fp32, CUDA cores + mma.sync, blocks of 16)
//   (KS|QS)^T = St [K;Q]^T                     (tcgen05, A = bf16 St from TMEM, right after
//                                               the state is read: overlaps A/P and the inverse)
//   Vn^T  = V^T T~^T + V^T Bl - (KS e^gamma)^T T~^T   (U - W S with W S =
//           T diag(beta e^gamma) (K S) = T~ diag(e^gamma) (K S), one tcgen05 accumulator;
//           T~ = T diag(beta) with the diagonal beta rounded to bf16, Bl = diag(beta -
//           bf16(beta)), so beta V enters with ~2^-17 relative error; the e^gamma row
//           scaling of K S is applied while K S is converted to a bf16 operand)
//   O^T   = scale (e^{gamma_t} (QS)^T + Vn^T P^T)   (tcgen05, A = bf16 Vn^T from TMEM)
//   St   <- e^{gamma_63} St + Vd^T K,  Vd = e^{gamma_63 - gamma_t} Vn as bf16 hi + lo (two
//           MMAs with A from TMEM) so the state update keeps ~16 mantissa bits.
// Everything after the state read works on transposed ([v][t]) accumulators,
// so every TMEM lane is a v row: each thread owns one v row of every
// accumulator, and the operands the threads produce (bf16 St, K S, Vn, Vd)
// go back to TMEM as tcgen05 A operands instead of through shared memory.
// Tokens past the end of the sequence get beta = 0 and log-decay 0, which
// makes their Vn rows exactly zero and leaves gamma_63 = gamma_{L-1}.
//
// Warp roles: warps 0-15 do the CUDA-core work (four per TMEM lane quarter,
// each on a quarter of the columns); warp 16 issues every TMA load and tcgen05
// MMA.  The two sides hand off through mbarriers only, so the tensor pipe runs
// St [K;Q]^T during the A/P phase, [K;Q]K^T of the next chunk during the Vn
// drain and the state update during the output epilogue.
// Math: same chunked algebra as cuda_kkt_inv_uw_v1.cu:1-20 (U, W, g_cu),
// cuda_h_v2b.cu (state scan) and cuda_o_v1.cu (output); semantics as
// definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:62-142.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_sm100.cuh"

namespace gdn {

__device__ uint32_t g_gdn_status = 0;

namespace {
using namespace sm100;

constexpr int kComputeWarps = 16;  // four per TMEM lane quarter
constexpr int kComputeThreads = 32 * kComputeWarps;
constexpr int kThreads = kComputeThreads + 32;  // + the TMA / MMA issue warp
constexpr uint32_t kComputeBar = 1;             // named barrier of the compute warps
constexpr int kL0Warp = 14;                     // warps 14-15 run the level-0 inverse
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait, then give up

// ---- shared memory map (offsets from a 1024-aligned base) -----------------
// Operand tiles are stacks of 128-byte rows in the SWIZZLE_128B pattern.
constexpr uint32_t kKQStage = 32768;  // [kb 2][row 128: K rows 0-63, Q rows 64-127][128 B]
constexpr uint32_t kVStage = 16384;   // [vb 2][t 64][128 B]
constexpr uint32_t OFF_KQ = 0;                     // 2 stages
constexpr uint32_t OFF_V = OFF_KQ + 2 * kKQStage;  // 2 stages
constexpr uint32_t OFF_P = OFF_V + 2 * kVStage;    // P: [t 64][128 B] (K-major B of Vn^T P^T)
constexpr uint32_t OFF_TB = OFF_P + 8192;          // T~ = T_off diag(beta): row s = column s (MN-major B)
constexpr uint32_t OFF_BL = OFF_TB + 8192;         // diag(beta - bf16(beta)), same layout (zero
                                                   // off the diagonal: cleared once per CTA)
constexpr int kAtPitch = 72;   // fp32 row pitch of A^T (72 = 8 mod 32: conflict-free tf32 A fragments)
constexpr int kTcPitch = 68;   // fp32 row pitch of T^T (68 = 4 mod 32: conflict-free B fragments)
constexpr uint32_t OFF_AT = OFF_BL + 8192;                // fp32 A^T [64][72]
constexpr uint32_t OFF_TC = OFF_AT + 64 * kAtPitch * 4;   // fp32 T^T [64][68]
constexpr uint32_t OFF_MC = OFF_TC + 64 * kTcPitch * 4;   // fp32 (A21 T11)^T [32][36]
constexpr uint32_t OFF_XC = OFF_MC + 32 * 36 * 4;         // fp32 level-1 products, 2 x [16][20]
constexpr uint32_t OFF_MC2 = OFF_XC + 2 * 320 * 4;        // second K-half of (A21 T11), columns 0-15
constexpr uint32_t OFF_TC2 = OFF_MC2 + 32 * 36 * 4;       // second K-half of T rows 48-63, cols 0-31 [32][20]
constexpr uint32_t OFF_O = (OFF_TC2 + 32 * 20 * 4 + 1023) / 1024 * 1024;  // output tile
// [cb 2][t 64][128 B] (TMA store source; written by the output epilogue, stored
// by the issue thread once the next chunk's T tiles are signalled)
constexpr uint32_t OFF_MISC = OFF_O + 16384;
// The final state passes through per-warp transpose tiles laid over the inverse's
// scratch (free after the last chunk): 32 rows x 16 floats at a pitch of 20
// floats, so that both the per-lane row writes and the row-segment reads are
// 16-byte accesses with the fewest bank wavefronts.
constexpr int kXposePitch = 20;
constexpr int kXposeFloats = 32 * kXposePitch;
static_assert(OFF_AT + 16 * kXposeFloats * 4 <= OFF_O, "transpose tiles overlap the output tile");
// the initial state staged by TMA (4 x 16 KiB, 1024-byte aligned for the swizzle)
// over the inverse's scratch and the output tile, both free before the first chunk
static_assert(OFF_AT % 1024 == 0 && OFF_AT + 65536 <= OFF_MISC, "staged state tile");
// Per-token tables of one chunk (floats), double-buffered by chunk parity.
constexpr int G_GAM = 0;     // gamma_t * log2(e) (cumulative log-decay)
constexpr int G_BET = 64;    // beta_t (0 past the end of the sequence)
constexpr int G_D = 128;     // 2^(gamma_t - gamma_{t-1}): per-token decay factor (1 past the end)
constexpr int G_DEC = 192;   // 2^(gamma_63 - gamma_t) for valid tokens, else 0
constexpr int G_EG = 256;    // scale * 2^gamma_t
constexpr int G_E2 = 320;    // 2^gamma_t
constexpr int G_RK = 384;    // 1 / |k_t| (q/k L2 norm only)
constexpr int G_RQ = 448;    // 1 / |q_t| (q/k L2 norm only)
constexpr int kGateFloats = 512;
constexpr uint32_t kMiscBarOff = 2 * kGateFloats * 4;  // barriers after both table buffers
constexpr uint32_t kSmemBytes = OFF_MISC + kMiscBarOff + 256 + 1024;  // + slack for the 1024 alignment

// ---- TMEM columns (every accumulator has lanes = v, except D1) -------------
constexpr uint32_t TM_ST = 0;     // St [v][k] fp32
constexpr uint32_t TM_KQS = 128;  // [K S | Q S]^T fp32: cols 0-63 (KS)^T[v][s], 64-127 (QS)^T[v][t]
constexpr uint32_t TM_D1 = 256;   // [K;Q] K^T fp32 [128 rows][64]
constexpr uint32_t TM_VN = 320;   // Vn^T fp32 [v][t], then (P Vn)^T [v][t]
constexpr uint32_t TM_SB = 384;   // A operand: St as bf16 [v][k] (64 cols), then
constexpr uint32_t TM_VDH = 384;  //   Vd_hi^T bf16 [v][t] (32 cols)
constexpr uint32_t TM_VDL = 416;  //   Vd_lo^T bf16 [v][t] (32 cols)
constexpr uint32_t TM_KSB = 448;  // A operand: (KS)^T bf16 [v][s] (32 cols), then
constexpr uint32_t TM_VNB = 448;  //   Vn^T bf16 [v][s] (32 cols)
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kTmaBytes = 2 * kKQStage / 2 + kVStage;  // K 16K + Q 16K + V 16K

// mbarriers (OFF_MISC + kMiscBarOff): TMA stages, tensor pipe -> compute warps
// (one tcgen05.commit each), compute warps -> issue warp (one arrive per warp;
// RDY_T1: warps 12-15, once the T~ rows 32-63 are written).
enum : int {
  BAR_TMA0 = 0, BAR_TMA1, BAR_M1, BAR_KQS, BAR_M3, BAR_PV, BAR_ST,
  RDY_S, RDY_T, RDY_V, BAR_END, RDY_T1, BAR_STATE, kNumBars
};

struct ChunkParams {
  const float* state;
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* a;
  const __nv_bfloat16* b;
  const int64_t* cu_seqlens;
  __nv_bfloat16* out;
  float* new_state;
  float* debug;  // optional dump of one chunk's intermediates
  const SegJob* jobs;  // segmented prefill: job table (nullptr: sequences from cu_seqlens)
  float scale;
  int tma_out;   // output rows of full chunks go through a TMA store (out is 16-byte aligned)
  int Hv_out, head_off;  // heads of the output buffer(s), position of this call's heads
  int n_peers;           // peer buffers that receive the same output rows
  __nv_bfloat16* peer_out[kMaxPeers];
  int64_t T, N;
  int Hq, Hv;
  int dbg_seq, dbg_head, dbg_chunk;
};

// A call of more (sequence, head) pairs than SMs runs in waves, and the CTA
// scheduler hands out CTAs in index order: with the longest sequences first,
// the short ones fill in behind them instead of a long one starting last
// (longest-processing-time order, by chunk count).  The ORDER instantiation does
// this; one warp ranks up to 64 sequences.
constexpr int kOrderMaxSeqs = 64;

// Tensor maps of the peer output buffers (n_peers used).
struct PeerMaps {
  CUtensorMap m[kMaxPeers];
};

constexpr int kClkSlots = 20;  // phase clock slots per compute warp (debug build)
// Debug dump layout (floats); the DBG_U block is not written (U is never formed
// on its own: the kernel computes V^T T~^T - (KS e^gamma)^T T~^T in one accumulator).
constexpr int DBG_GAM = 0, DBG_BET = 64, DBG_A = 128, DBG_P = DBG_A + 4096, DBG_T = DBG_P + 4096,
              DBG_U = DBG_T + 4096, DBG_KS = DBG_U + 8192, DBG_VN = DBG_KS + 8192,
              DBG_QS = DBG_VN + 8192, DBG_PV = DBG_QS + 8192, DBG_ST = DBG_PV + 8192,
              DBG_CLK = DBG_ST + 16384, DBG_MCLK = DBG_CLK + 16 * kClkSlots, DBG_EV = DBG_MCLK + 16,
              DBG_SIZE = DBG_EV + 96;
// DBG_CLK: [warp 16][kClkSlots] SM cycles lane 0 of each compute warp of the
// debug CTA spent in each phase, summed over all chunks of its sequence
// (phases: the PHASE() marks in the chunk loop); DBG_MCLK: the same for the
// issue thread (MPHASE() marks).  DBG_EV: SM-clock timestamps (from a common
// base) of handoff events around chunk dbg_chunk + 2 (away from the dump's own
// stores): [warp 16][5] for the compute warps, then 8 for the issue thread.

// 16 consecutive floats of a per-token table (16-byte aligned) as four vector loads
// Two fp32 lanes per instruction (sm_100 packed FMUL2 / FFMA2 / FADD2); each
// lane rounds exactly like the scalar operation.
__device__ __forceinline__ float2 mul2(float a0, float a1, float b0, float b1) {
  return __fmul2_rn(make_float2(a0, a1), make_float2(b0, b1));
}

__device__ __forceinline__ void load_table16(const float* src, float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = reinterpret_cast<const float4*>(src)[q];
    v[4 * q] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
}

// The final state of one warp's 32 x 32 block (rows = TMEM lanes of the warp's
// quarter, 32 columns from tq) to HBM, coalesced: each half of 16 columns passes
// from the lane that owns the row through the warp's transpose tile in shared
// memory, and lane l stores rows 8 j + l / 4 at column 4 (l % 4) in 16-byte
// pieces (a warp instruction covers eight 64-byte row segments).  Each lane
// storing its own row puts 32 rows 512 bytes apart in every instruction, one
// transaction per lane (~2 us per CTA).  Kept out of line: the chunk loop's code
// is sensitive to what surrounds it (the same treatment of the initial-state load,
// as a call before the loop, slowed the loop by 1.5 %).
__device__ __noinline__ void state_from_tmem(float* blk, float* scr, uint32_t tq, int lane) {
  float v[32];
  tmem_ld32(tq, v);
  tmem_wait_ld();
  reg_fence(v);
  const int r0 = lane >> 2, c0 = 4 * (lane & 3);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<float4*>(scr + lane * kXposePitch + 4 * k) =
          make_float4(v[16 * hf + 4 * k], v[16 * hf + 4 * k + 1], v[16 * hf + 4 * k + 2],
                      v[16 * hf + 4 * k + 3]);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j)
      st_stream_f4(blk + (8 * j + r0) * kHead + 16 * hf + c0,
                   *reinterpret_cast<const float4*>(scr + (8 * j + r0) * kXposePitch + c0));
    __syncwarp();  // read before the next half is written
  }
}

// ORDER: lane i of the calling warp takes sequences i and i + 32 (N <= 64) with
// the key (chunks << 6) | (63 - index), unique, so that more chunks rank first and
// equal counts keep their order (lengths clamped as the chunk loop clamps them);
// the rank of a sequence is the number of larger keys.  The sequence of rank n
// and its bounds go to *seq_slot and seq_bounds[0..1].  Kept out of line (one
// call per CTA): inlined, the ordered calls ran up to 1.3 % slower.  All four
// loads are issued at once, and four partial counts keep the additions
// independent.
__device__ __noinline__ void rank_longest_first(const int64_t* cu, int ns, int64_t T, int64_t n,
                                                int lane, int* seq_slot, int64_t* seq_bounds) {
  // indices clamped into cu[0..ns]; the values of lanes past ns are not used
  int64_t c[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) c[u] = cu[min(lane + 32 * (u >> 1) + (u & 1), ns)];
  int64_t b[2], e[2];
  int key[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    b[u] = min(max(c[2 * u], int64_t(0)), T);
    e[u] = min(max(c[2 * u + 1], b[u]), T);
    key[u] = lane + 32 * u < ns
                 ? static_cast<int>(((e[u] - b[u] + kChunk - 1) / kChunk) << 6) | (63 - lane - 32 * u)
                 : -1;
  }
  int r0[4] = {0, 0, 0, 0}, r1[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int kj = __shfl_sync(0xffffffffu, key[0], j);
    r0[j & 3] += kj > key[0] ? 1 : 0;
    r1[j & 3] += kj > key[1] ? 1 : 0;
  }
  if (ns > 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int kj = __shfl_sync(0xffffffffu, key[1], j);
      r0[j & 3] += kj > key[0] ? 1 : 0;
      r1[j & 3] += kj > key[1] ? 1 : 0;
    }
  }
  const int q0 = r0[0] + r0[1] + r0[2] + r0[3], q1 = r1[0] + r1[1] + r1[2] + r1[3];
  const int u = (key[0] >= 0 && q0 == n) ? 0 : (key[1] >= 0 && q1 == n) ? 1 : -1;  // exactly one
  if (u >= 0) {
    *seq_slot = lane + 32 * u;
    seq_bounds[0] = b[u];
    seq_bounds[1] = e[u];
  }
}

// L2: q/k L2 norm folded in as per-token factors; JOBS: the segmented prefill's
// job table (identity start, v = 0, no outputs, optional final state); ORDER
// (without JOBS): CTA group r runs the r-th longest sequence; STAGED (without
// JOBS, a given initial state): the issue thread brings the initial state tile
// into shared memory by TMA (tm_s).  All are separate instantiations so the plain
// kernel carries none of it (as a runtime switch, the staging slowed the chunk
// loop of every call by ~2.4 %).
template <bool DEBUG, bool L2, bool JOBS, bool ORDER, bool STAGED>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_prefill_chunked_kernel(const __grid_constant__ CUtensorMap tm_q,
                               const __grid_constant__ CUtensorMap tm_k,
                               const __grid_constant__ CUtensorMap tm_v,
                               const __grid_constant__ CUtensorMap tm_o,
                               const __grid_constant__ CUtensorMap tm_s,
                               const __grid_constant__ PeerMaps pm, const ChunkParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align by offsetting the __shared__ array itself (not through an integer
  // cast), so every derived pointer stays in the shared state space and its
  // accesses compile to ld/st.shared rather than generic loads and stores.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  // per-token gate tables (G_*), double-buffered by chunk parity: the tables
  // of chunk c+1 are computed while chunk c's tensor-core work runs.
  float* gates_buf = reinterpret_cast<float*>(smem + OFF_MISC);  // [2][kGateFloats]
  float* At = reinterpret_cast<float*>(smem + OFF_AT);   // A column-major: At[k][i] = A[i][k]
  float* Tcm = reinterpret_cast<float*>(smem + OFF_TC);  // Tcm[j][i] = T[i][j]
  float* Mcm = reinterpret_cast<float*>(smem + OFF_MC);  // (A21 T11) column-major, pitch 36
  float* Xcm = reinterpret_cast<float*>(smem + OFF_XC);  // 2 x [16][20] level-1 products
  float* Mcm2 = reinterpret_cast<float*>(smem + OFF_MC2);  // second K-half of M (columns 0-15)
  float* Tcm2 = reinterpret_cast<float*>(smem + OFF_TC2);  // second K-half of T[48:64][0:32]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3;    // TMEM lane quarter this warp may access
  const int cq = (warp >> 2) & 3;  // column quarter handled by this warp
  const int g = lane >> 2, tq = lane & 3;  // mma.sync fragment coordinates
  const int rowv = 32 * quarter + lane;    // TMEM lane (accumulator row) of this thread
  const int h = static_cast<int>(blockIdx.x % p.Hv);
  int64_t n = blockIdx.x / p.Hv;
  const int qh = h / (p.Hv / p.Hq);
  constexpr int64_t kStateFloats = kHead * kHead;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_MISC + kMiscBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile uint32_t* abort_flag = tmem_slot + 1;  // a compute thread gave up on a wait
  int* seq_slot = reinterpret_cast<int*>(tmem_slot + 2);  // sequence of this CTA group (ORDER)
  int64_t* seq_bounds = reinterpret_cast<int64_t*>(tmem_slot + 4);  // its [bos, eos)

  // Barriers, tensor-map prefetch and the TMEM allocation, then a CTA barrier.
  auto setup = [&]() {
    if (tid == 0) {
      for (int i = 0; i < kNumBars; ++i)
        mbar_init(&bars[i], (i >= RDY_S && i <= RDY_V) ? kComputeWarps : i == RDY_T1 ? 4 : 1);
      fence_mbar_init();
      *abort_flag = 0u;
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      if (p.tma_out) prefetch_tmap(&tm_o);
      if (STAGED) prefetch_tmap(&tm_s);
    }
    if (warp == 0) {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };

  int64_t bos, eos;
  if constexpr (ORDER) {
    // warp 1 finds the sequence of rank n while warp 0 sets up; the bounds it
    // read come along, so no second load of cu_seqlens follows
    if (warp == 1) rank_longest_first(p.cu_seqlens, static_cast<int>(p.N), p.T, n, lane, seq_slot, seq_bounds);
    setup();
    // (clamped again, so that every access stays in bounds whatever the slot held)
    n = min(max(static_cast<int64_t>(*seq_slot), int64_t(0)), p.N - 1);
    bos = min(max(seq_bounds[0], int64_t(0)), p.T);
    eos = min(max(seq_bounds[1], bos), p.T);
  }

  const float* state_in;  // this head's initial state (nullptr: zero)
  float* ns_rows;         // this head's final state (nullptr: not stored)
  uint32_t jflags = 0;
  if constexpr (JOBS) {  // one segment of a sequence (job values are written on the device)
    const SegJob jb = p.jobs[n];
    bos = min(max(jb.bos, int64_t(0)), p.T);
    eos = min(max(jb.eos, bos), p.T);
    state_in = jb.state_in ? jb.state_in + h * kStateFloats : nullptr;
    ns_rows = jb.state_out ? jb.state_out + h * kStateFloats : nullptr;
    jflags = jb.flags;
  } else {
    if constexpr (!ORDER) {
      bos = min(max(p.cu_seqlens[n], int64_t(0)), p.T);
      eos = min(max(p.cu_seqlens[n + 1], bos), p.T);
    }
    state_in = p.state ? p.state + (n * p.Hv + h) * kStateFloats : nullptr;
    ns_rows = p.new_state + (n * p.Hv + h) * kStateFloats;
  }
  const int64_t Ltot = eos - bos;
  const bool init_identity = JOBS && (jflags & kJobIdentity);
  const bool v_zero = JOBS && (jflags & kJobNoV);
  const bool write_out = !JOBS || !(jflags & kJobNoOut);

  if (Ltot <= 0) {  // empty sequence: zero final state (definition skips it)
    if (ns_rows)
      for (int i = tid; i < kHead * kHead / 4; i += kThreads)
        reinterpret_cast<float4*>(ns_rows)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (ORDER) {
      if (warp == 0) tmem_dealloc(*tmem_slot, kTmemCols);
    }
    return;
  }
  const int nchunks = static_cast<int>((Ltot + kChunk - 1) / kChunk);

  if constexpr (!ORDER) setup();
  const uint32_t tmem = *tmem_slot;
  const long long t_base = DEBUG ? clock64() : 0;
  bool failed = false;  // this thread gave up on a wait

  if (warp < kComputeWarps) {
    // ======================= compute warps =================================
    const bool dbg_cta = DEBUG && p.debug && n == p.dbg_seq && h == p.dbg_head;
    long long clk_acc[kClkSlots];
    long long clk_last = 0;
    if constexpr (DEBUG) {
#pragma unroll
      for (int i = 0; i < kClkSlots; ++i) clk_acc[i] = 0;
      clk_last = clock64();
    }
#define PHASE(k)                              \
  if constexpr (DEBUG) {                      \
    const long long now_ = clock64();         \
    clk_acc[k] += now_ - clk_last;            \
    clk_last = now_;                          \
  }
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tq_st = tmem + lane_base + TM_ST + 32 * cq;  // this thread's St columns
    const float neg_exp_A = -expf(p.A_log[h]);
    const float dt_bias_h = p.dt_bias[h];

    // One arrival per warp on a compute -> issue-warp barrier after this
    // thread's TMEM operand stores (waited), optionally with its shared-memory
    // operand writes made visible to the async proxy first.
    auto signal = [&](int b, bool smem_written) {
      if (smem_written) fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[b]);
    };
    // Bounded wait on a tensor-pipe commit.  After a timeout the thread stops
    // waiting and runs on (its results are then garbage, the status word says
    // so); the compute warps agree once per chunk to leave the loop.
    auto wait_mma = [&](int b, uint32_t parity) {
      if (!failed) failed = !mbar_wait_nap(&bars[b], parity, kTimeoutNs);
      tc_fence_after();
    };

    // Gates of one chunk from raw a/b values held by warp 1 (two tokens per lane):
    // log-decay, its inclusive scan (gamma, stored in log2 units), beta and the
    // derived per-token tables.
    // raw bf16 bits: nothing consumes a prefetched value until the next
    // compute_gates, so the global loads stay in flight meanwhile
    unsigned short ga_raw[2] = {0, 0}, gb_raw[2] = {0, 0};
    auto prefetch_gates = [&](int cc) {
      const int64_t t0c = bos + static_cast<int64_t>(cc) * kChunk;
      const unsigned short* pa = reinterpret_cast<const unsigned short*>(p.a);
      const unsigned short* pb = reinterpret_cast<const unsigned short*>(p.b);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t t = t0c + 2 * lane + e;
        if (t < eos) {
          ga_raw[e] = pa[t * p.Hv + h];
          gb_raw[e] = pb[t * p.Hv + h];
        }
      }
    };
    auto compute_gates = [&](int cc) {  // warp 1 only
      const int64_t t0c = bos + static_cast<int64_t>(cc) * kChunk;
      const int Lc = static_cast<int>(min(static_cast<int64_t>(kChunk), eos - t0c));
      float lg[2], bt[2];
      bool valid[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        valid[e] = 2 * lane + e < Lc;
        lg[e] = valid[e] ? neg_exp_A * softplus_t20_fast(bf16_bits_to_f32(ga_raw[e]) + dt_bias_h) : 0.f;
        bt[e] = valid[e] ? sigmoid_fast(bf16_bits_to_f32(gb_raw[e])) : 0.f;
      }
      const float pair = lg[0] + lg[1];
      float incl = pair;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += y;
      }
      const float gt[2] = {(incl - pair + lg[0]) * kLog2e, incl * kLog2e};
      const float g63 = __shfl_sync(0xffffffffu, gt[1], 31);
      float* gb = gates_buf + (cc & 1) * kGateFloats;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * lane + e;
        const float eg = ex2_ftz(gt[e]);
        gb[G_GAM + t] = gt[e];
        gb[G_BET + t] = bt[e];
        gb[G_D + t] = ex2_ftz(lg[e] * kLog2e);
        gb[G_DEC + t] = valid[e] ? ex2_ftz(g63 - gt[e]) : 0.f;
        gb[G_EG + t] = p.scale * eg;
        gb[G_E2 + t] = eg;
      }
    };
    auto dump_state = [&]() {  // debug: St after the state update of the debug chunk
      float v[32];
      tmem_ld32(tq_st, v);
      tmem_wait_ld();
      reg_fence(v);
      for (int i = 0; i < 32; ++i) p.debug[DBG_ST + rowv * 128 + 32 * cq + i] = v[i];
    };

    // q/k L2 norm: 1 / sqrt(sum x^2 + 1e-6) of every K and Q row of chunk cc's
    // stage (rows 0-63 K, 64-127 Q; a row's 64 elements of a 128-byte line are
    // permuted by the swizzle, which a sum of squares ignores), four threads per
    // row.  The factors scale A/P columns and rows, K S columns, Vd rows and the
    // Q S columns of the output instead of the operands themselves.
    auto qk_norms = [&](int cc) {
      const int r = tid >> 2, part = tid & 3;
      const uint32_t base = sb + OFF_KQ + (cc & 1) * kKQStage + r * 128 + part * 32;
      float acc = 0.f;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint4 w = lds128(base + kb * 16384 + hh * 16);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16_lo(ws[e]), hi = bf16_hi(ws[e]);
            acc = fmaf(lo, lo, fmaf(hi, hi, acc));
          }
        }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (part == 0) gates_buf[(cc & 1) * kGateFloats + (r < 64 ? G_RK + r : G_RQ + r - 64)] = rsqrtf(acc + 1e-6f);
    };

    if (warp == 1) prefetch_gates(0);  // in flight during the state load

    // ---- initial state -> TMEM (row rowv, columns [32 cq, 32 cq + 32)) -----
    {
      const float* src = state_in && !init_identity ? state_in + rowv * kHead + 32 * cq : nullptr;
      float v[32];
      if constexpr (STAGED) {
        // the issue thread loads the tile by TMA, columns [32 c, 32 c + 32) at
        // OFF_AT + 16 KiB c in the 128-byte swizzle, so this thread's eight
        // 16-byte pieces of row rowv come from shared memory (four wavefronts per
        // warp read, the fewest) instead of 512-byte-strided global loads (one
        // transaction per lane)
        wait_mma(BAR_STATE, 0u);
        const uint32_t srow = sb + OFF_AT + cq * 16384 + rowv * 128;
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const uint4 w = lds128(srow + ((q4 ^ (rowv & 7)) << 4));
          v[4 * q4] = __uint_as_float(w.x);
          v[4 * q4 + 1] = __uint_as_float(w.y);
          v[4 * q4 + 2] = __uint_as_float(w.z);
          v[4 * q4 + 3] = __uint_as_float(w.w);
        }
      } else {
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          float4 x = src ? ld_stream_f4(src + q4 * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[4 * q4] = x.x;
          v[4 * q4 + 1] = x.y;
          v[4 * q4 + 2] = x.z;
          v[4 * q4 + 3] = x.w;
        }
      }
      if (init_identity) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = (rowv == 32 * cq + i) ? 1.f : 0.f;
      }
      tmem_st32(tq_st, v);
      tmem_wait_st();
    }

    if (warp == 1) {
      compute_gates(0);
      if (Ltot > kChunk) prefetch_gates(1);
    }
    for (int i = tid; i < 8192 / 16; i += kComputeThreads)  // Bl: zero off the diagonal
      sts128(sb + OFF_BL + 16 * i, 0u, 0u, 0u, 0u);
    if (v_zero) {  // no V loads: both V stages hold zeros for the whole sequence
      for (int i = tid; i < 2 * kVStage / 16; i += kComputeThreads)
        sts128(sb + OFF_V + 16 * i, 0u, 0u, 0u, 0u);
      fence_async_smem();
    }
    if constexpr (L2) {  // chunk 0's factors, published by the first loop-top barrier
      wait_mma(BAR_M1, 0u);
      qk_norms(0);
    }
    bool aborted = false;

    for (int c = 0; c < nchunks; ++c) {
      const int stage = c & 1;
      const uint32_t par = static_cast<uint32_t>(c & 1);
      const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
      const int L = static_cast<int>(min(static_cast<int64_t>(kChunk), eos - t0));
      const bool dbg = dbg_cta && c == p.dbg_chunk;

      // previous chunk's state update done: St is final and its TMEM operands
      // are free.  The barrier also publishes this chunk's gates (warp 1).
      if (c > 0) {  // the state update is the next step on the chain: poll it closely
        bool done = false;
#pragma unroll 1
        for (int i = 0; i < 256 && !done; ++i) done = mbar_test(&bars[BAR_ST], par ^ 1u);
        if (!done) wait_mma(BAR_ST, par ^ 1u);
        tc_fence_after();
      }
      PHASE(17)
      if (DEBUG && dbg_cta && c == p.dbg_chunk + 3 && lane == 0)
        p.debug[DBG_EV + warp * 5 + 3] = float(clock64() - t_base);
      if (failed) *abort_flag = 1u;
      named_sync(kComputeBar, kComputeThreads);
      if (*abort_flag) { aborted = true; break; }
      if (DEBUG && dbg_cta && c == p.dbg_chunk + 3 && lane == 0)
        p.debug[DBG_EV + warp * 5 + 4] = float(clock64() - t_base);
      if (dbg_cta && c - 1 == p.dbg_chunk) dump_state();
      PHASE(0)

      const float* gam = gates_buf + stage * kGateFloats + G_GAM;
      const float* bet = gam + G_BET;
      if (dbg && tid < 64) {
        p.debug[DBG_GAM + tid] = gam[tid] / kLog2e;
        p.debug[DBG_BET + tid] = bet[tid];
      }
      PHASE(1)

      // ---- state pass: St -> bf16 A operand in TMEM; St *= e^{gamma_63} ----
      {
        const float dec = ex2_ftz(gam[63]);
        float v[32];
        tmem_ld32(tq_st, v);
        tmem_wait_ld();
        reg_fence(v);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
        tmem_st16u(tmem + lane_base + TM_SB + 16 * cq, w);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 r = mul2(v[i], v[i + 1], dec, dec);
          v[i] = r.x;
          v[i + 1] = r.y;
        }
        tmem_st32(tq_st, v);
        tmem_wait_st();
      }
      if (tid < 64) {  // Bl: beta_j - bf16(beta_j) on the diagonal (row j, column j)
        const int j = tid;
        const float blo = bet[j] - bf16_lo(pack_bf16x2(bet[j], 0.f));
        const uint32_t w = pack_bf16x2(blo, 0.f);  // bf16(blo) in the low half
        sts32(sb + OFF_BL + sw128_off(j, j >> 3) + 4 * ((j & 7) >> 1), (j & 1) ? (w << 16) : w);
      }
      signal(RDY_S, tid < 64);  // the tensor pipe reads Bl right after the state
      PHASE(2)
      wait_mma(BAR_M1, par);
      PHASE(3)

      // ---- A (rows 0-63 of D1: quarters 0-1, stored column-major) and
      //      P (rows 64-127: quarters 2-3) -----------------------------------
      {
        const int i = rowv & 63;
        const float gi = gam[i];
        float v[16];
        tmem_ld16(tmem + lane_base + TM_D1 + 16 * cq, v);
        tmem_wait_ld();
        reg_fence(v);
        PHASE(4)
        if constexpr (L2) {  // A[i][j] / (|k_i| |k_j|), P[i][j] / (|q_i| |k_j|)
          float rc[16];
          load_table16(gam + G_RK + 16 * cq, rc);
          const float rr = quarter < 2 ? gam[G_RK + i] : gam[G_RQ + i];
#pragma unroll
          for (int jj = 0; jj < 16; jj += 2) {
            const float2 x = mul2(v[jj], v[jj + 1], rc[jj] * rr, rc[jj + 1] * rr);
            v[jj] = x.x;
            v[jj + 1] = x.y;
          }
        }
        // e^{gamma_i - gamma_j} for this block's 16 columns, walking down each
        // group of 4 from its highest column j <= i with e(j-1) = e(j) d_j,
        // d_j = e^{gamma_j - gamma_{j-1}} <= 1: one ex2 per group, the rest on
        // the FMA pipe, and no overflow whatever the decay (columns above the
        // diagonal are masked).
        const int r0 = 16 * cq;
        float dd[16];
        load_table16(gam + G_D + r0, dd);
        float ef[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // four independent 4-column chains
          const int top = r0 + 4 * q + 3;
          float e = (top <= i) ? ex2_ftz(gi - gam[top]) : 1.f;
#pragma unroll
          for (int jj = 4 * q + 3; jj >= 4 * q; --jj) {
            ef[jj] = e;
            e = (r0 + jj > i) ? 1.f : e * dd[jj];
          }
        }
        if (quarter < 2) {
          const float bi = bet[i];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = r0 + jj;
            const float aij = (j < i) ? bi * v[jj] * ef[jj] : 0.f;
            At[j * kAtPitch + i] = aij;
            if (dbg) p.debug[DBG_A + i * 64 + j] = aij;
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = r0 + jj;
            v[jj] = (j <= i) ? v[jj] * ef[jj] : 0.f;
          }
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2)
            sts128(sb + OFF_P + sw128_off(i, 2 * cq + c2), pack_bf16x2(v[8 * c2], v[8 * c2 + 1]),
                   pack_bf16x2(v[8 * c2 + 2], v[8 * c2 + 3]), pack_bf16x2(v[8 * c2 + 4], v[8 * c2 + 5]),
                   pack_bf16x2(v[8 * c2 + 6], v[8 * c2 + 7]));
          if (dbg)
            for (int jj = 0; jj < 16; ++jj) p.debug[DBG_P + i * 64 + r0 + jj] = v[jj];
        }
      }
      PHASE(5)
      named_sync(kComputeBar, kComputeThreads);
      PHASE(6)

      // ---- (KS)^T -> bf16 A operand of the Vn MMAs: lanes v, 16-token column
      //      groups; warps 10-11 also convert the groups of warps 14-15, which
      //      run the level-0/1 inverse meanwhile.
      auto convert_ks = [&](int grp) {
        float v[16];
        tmem_ld16(tmem + lane_base + TM_KQS + 16 * grp, v);
        float e2[16];  // 2^g_s of these 16 tokens
        load_table16(gam + G_E2 + 16 * grp, e2);
        if constexpr (L2) {  // K S columns / |k_s|
          float rk[16];
          load_table16(gam + G_RK + 16 * grp, rk);
#pragma unroll
          for (int e = 0; e < 16; ++e) e2[e] *= rk[e];
        }
        tmem_wait_ld();
        reg_fence(v);
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 r = mul2(v[2 * e], v[2 * e + 1], e2[2 * e], e2[2 * e + 1]);
          w[e] = pack_bf16x2(r.x, r.y);
        }
        tmem_st8u(tmem + lane_base + TM_KSB + 8 * grp, w);
        if (dbg)
          for (int i = 0; i < 16; ++i) p.debug[DBG_KS + (16 * grp + i) * 128 + rowv] = v[i];
      };

      // ---- T = (I + A)^-1, fp32, blocks of 16:
      //      level 0: the four diagonal blocks by right-looking elimination and
      //      level 1: T10 = -T11 A10 T00 (warp 14), T32 = -T33 A32 T22 (warp 15),
      //      each warp on its own blocks (mma.sync, warp-local);
      //      level 2: [T20 T21; T30 T31] = -T22' (A21' T11'), primes = 32x32 halves.
      if (warp < kL0Warp) {
        wait_mma(BAR_KQS, par);
        convert_ks(cq);
        if (cq == 2 && quarter >= 2) convert_ks(3);
        tmem_wait_st();
        tc_fence_before();  // read by the Vn MMAs after the next barrier
        if (warp == 1 && c + 1 < nchunks) {  // gates of the next chunk (published by
          compute_gates(c + 1);              // the next loop-top barrier)
          if (c + 2 < nchunks) prefetch_gates(c + 2);
        }
      } else {
        const int u = tid - 32 * kL0Warp;
        const int b = u >> 4, j = u & 15, b0 = 16 * b;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) x[r] = (r == j) ? 1.f : 0.f;
#pragma unroll
        for (int k = 0; k < 15; ++k) {
          const float xk = x[k];
          const float* col = At + (b0 + k) * kAtPitch + b0;  // A[b0 + i][b0 + k]
#pragma unroll
          for (int q = (k + 1) / 4; q < 4; ++q) {
            const float4 a4 = *reinterpret_cast<const float4*>(col + 4 * q);
            if (4 * q + 0 > k) x[4 * q + 0] = fmaf(-a4.x, xk, x[4 * q + 0]);
            if (4 * q + 1 > k) x[4 * q + 1] = fmaf(-a4.y, xk, x[4 * q + 1]);
            if (4 * q + 2 > k) x[4 * q + 2] = fmaf(-a4.z, xk, x[4 * q + 2]);
            if (4 * q + 3 > k) x[4 * q + 3] = fmaf(-a4.w, xk, x[4 * q + 3]);
          }
        }
        float* tcol = Tcm + (b0 + j) * kTcPitch;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<float4*>(tcol + b0 + 4 * q) =
              make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
        for (int q = 0; q < 4 * b; ++q)  // rows above the diagonal block are zero
          *reinterpret_cast<float4*>(tcol + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
              __syncwarp();
        // level 1 of this warp's pair: X = A_IJ T_JJ, then T_IJ = -T_II X
        // (mma.sync m16n8k8, tf32; X through warp-private smem for the
        // fragment layout)
        const int pr = warp - kL0Warp;
        const int J0 = 32 * pr, I0 = J0 + 16;
        float* xw = Xcm + pr * 320;  // X column-major: X[r][j] at xw[j * 20 + r]
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        auto l1a_step = [&](float* acc, int nt, int k0) {
          const float* ar = At + (J0 + k0 + tq) * kAtPitch + I0 + g;           // A[I0+g][J0+k0+t]
          const float* br = Tcm + (J0 + 8 * nt + g) * kTcPitch + J0 + k0 + tq;  // T[J0+k0+t][J0+8nt+g]
          mma_tf32_16x8x8(acc, to_tf32(ar[0]), to_tf32(ar[8]), to_tf32(ar[4 * kAtPitch]),
                          to_tf32(ar[4 * kAtPitch + 8]), to_tf32(br[0]), to_tf32(br[4]));
        };
        l1a_step(c0, 0, 0);
        l1a_step(c0, 0, 8);
        l1a_step(c1, 1, 8);  // T_JJ[k][n] = 0 for k < n: columns 8-15 need k >= 8 only
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float* cc = nt ? c1 : c0;
          xw[(8 * nt + 2 * tq) * 20 + g] = cc[0];
          xw[(8 * nt + 2 * tq + 1) * 20 + g] = cc[1];
          xw[(8 * nt + 2 * tq) * 20 + g + 8] = cc[2];
          xw[(8 * nt + 2 * tq + 1) * 20 + g + 8] = cc[3];
        }
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          float dacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int k0 = 0; k0 < 16; k0 += 8) {
            const float* ar = Tcm + (I0 + k0 + tq) * kTcPitch + I0 + g;  // T[I0+g][I0+k0+t]
            const float* br = xw + (8 * nt + g) * 20 + k0 + tq;          // X[k0+t][8nt+g]
            mma_tf32_16x8x8(dacc, to_tf32(ar[0]), to_tf32(ar[8]), to_tf32(ar[4 * kTcPitch]),
                            to_tf32(ar[4 * kTcPitch + 8]), to_tf32(br[0]), to_tf32(br[4]));
          }
          float* tc = Tcm + (J0 + 8 * nt + 2 * tq) * kTcPitch + I0 + g;  // T[I0+r][J0+8nt+j]
          tc[0] = -dacc[0];
          tc[kTcPitch] = -dacc[1];
          tc[8] = -dacc[2];
          tc[kTcPitch + 8] = -dacc[3];
        }
      }
      named_sync(kComputeBar, kComputeThreads);
      PHASE(15)
      // T~ = T diag(beta) as a bf16 tile in which row j holds column j of T: the
      // MN-major B operand (K = s rows, N = t contiguous) of both V^T T~^T and
      // (KS e^gamma)^T T~^T.  Its diagonal is beta_j rounded to bf16; the
      // rounding remainder is on the diagonal of Bl (written with the state
      // pass).  One call writes the 16-byte chunk ch (T rows 8 ch .. 8 ch + 7)
      // of tile row j.  Rows 32-63 (columns 32-63 of T) are final after level
      // 1: warps 12-15 write them during level 2 and the tensor pipe takes the
      // Vn MMAs of those K rows early; rows 0-31 follow the last barrier.
      auto t_chunk = [&](int j, int ch) {
        const float sc = bet[j];
        const float* src = Tcm + j * kTcPitch + ch * 8;
        float4 x0 = *reinterpret_cast<const float4*>(src);
        float4 x1 = *reinterpret_cast<const float4*>(src + 4);
        if (j < 32 && ch >= 6) {  // T rows 48-63 of columns 0-31: add level 2's second K half
          const float* s2 = Tcm2 + j * 20 + 8 * (ch - 6);
          const float4 y0 = *reinterpret_cast<const float4*>(s2);
          const float4 y1 = *reinterpret_cast<const float4*>(s2 + 4);
          x0 = make_float4(x0.x + y0.x, x0.y + y0.y, x0.z + y0.z, x0.w + y0.w);
          x1 = make_float4(x1.x + y1.x, x1.y + y1.y, x1.z + y1.z, x1.w + y1.w);
        }
        const float2 r0 = mul2(x0.x, x0.y, sc, sc), r1 = mul2(x0.z, x0.w, sc, sc);
        const float2 r2 = mul2(x1.x, x1.y, sc, sc), r3 = mul2(x1.z, x1.w, sc, sc);
        sts128(sb + OFF_TB + sw128_off(j, ch), pack_bf16x2(r0.x, r0.y), pack_bf16x2(r1.x, r1.y),
               pack_bf16x2(r2.x, r2.y), pack_bf16x2(r3.x, r3.y));
      };
      if (warp >= 12) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int k = tid - 384 + 128 * r;  // 256 chunks of rows 32-63
          t_chunk(32 + (k >> 3), k & 7);
        }
        signal(RDY_T1, true);
      }
      // level 2 on the tensor cores (mma.sync m16n8k8, tf32 in, fp32 accumulate;
      // tf32 rounding, 2^-11, is below the bf16 rounding T gets right after).
      // Zero k-steps of the triangular factors are skipped and the longer
      // 16x8 output tiles are split over two warps by K half (at most two
      // dependent MMAs per warp); the second halves land in Mcm2 / Tcm2 and
      // are added where they are read.
      if (warp < 12) {  // step 1: M = A21' T11' (32x32x32), T11'[k][n] = 0 for k < n
        const int rt = warp / 6, u = warp % 6, t4 = tq;
        // (column tile, first k-step, k-steps, second half?) for u = 0..5
        const int ct = u < 2 ? 0 : u < 4 ? 1 : u - 2;
        const int ks0 = u == 0 ? 0 : u == 2 ? 1 : u == 5 ? 3 : 2;
        const int nks = (u == 2 || u == 5) ? 1 : 2;
        const bool second = (u == 1 || u == 3);
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2) {
          if (s2 < nks) {
            const int k0 = 8 * (ks0 + s2);
            const float* ar = At + (k0 + t4) * kAtPitch + 32 + 16 * rt + g;  // A[32+16rt+g][k0+t]
            const float* br = Tcm + (8 * ct + g) * kTcPitch + k0 + t4;       // T[k0+t][8ct+g]
            mma_tf32_16x8x8(cacc, to_tf32(ar[0]), to_tf32(ar[8]), to_tf32(ar[4 * kAtPitch]),
                            to_tf32(ar[4 * kAtPitch + 8]), to_tf32(br[0]), to_tf32(br[4]));
          }
        }
        float* mc = (second ? Mcm2 : Mcm) + (8 * ct + 2 * t4) * 36 + 16 * rt + g;  // M[r][j] at [j*36 + r]
        mc[0] = cacc[0];
        mc[36] = cacc[1];
        mc[8] = cacc[2];
        mc[36 + 8] = cacc[3];
      }
      named_sync(kComputeBar, kComputeThreads);
      PHASE(18)
      if (warp < 12) {  // step 2: T21' = -T22' M, T22'[r][k] = 0 for k > r
        const int t4 = tq;
        const int rt = warp < 4 ? 0 : 1;
        const int ct = warp < 4 ? warp : (warp - 4) >> 1;
        const int half = warp < 4 ? 0 : (warp - 4) & 1;  // rows 16-31 of T22': k-steps {0,1} or {2,3}
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2) {
          const int k0 = 8 * (2 * half + s2);
          const float* ar = Tcm + (32 + k0 + t4) * kTcPitch + 32 + 16 * rt + g;  // T[32+16rt+g][32+k0+t]
          const int mo = (8 * ct + g) * 36 + k0 + t4;                           // M[k0+t][8ct+g]
          float b0 = Mcm[mo], b1 = Mcm[mo + 4];
          if (ct < 2) {
            b0 += Mcm2[mo];
            b1 += Mcm2[mo + 4];
          }
          mma_tf32_16x8x8(cacc, to_tf32(ar[0]), to_tf32(ar[8]), to_tf32(ar[4 * kTcPitch]),
                          to_tf32(ar[4 * kTcPitch + 8]), to_tf32(b0), to_tf32(b1));
        }
        if (half == 0) {
          float* tc = Tcm + (8 * ct + 2 * t4) * kTcPitch + 32 + 16 * rt + g;  // T[32+r][j] at Tcm[j][32+r]
          tc[0] = -cacc[0];
          tc[kTcPitch] = -cacc[1];
          tc[8] = -cacc[2];
          tc[kTcPitch + 8] = -cacc[3];
        } else {
          float* tc = Tcm2 + (8 * ct + 2 * t4) * 20 + g;  // T[48+r][j] at Tcm2[j*20 + r]
          tc[0] = -cacc[0];
          tc[20] = -cacc[1];
          tc[8] = -cacc[2];
          tc[28] = -cacc[3];
        }
      }
      named_sync(kComputeBar, kComputeThreads);
      PHASE(7)
      if (tid < 256) t_chunk(tid & 31, tid >> 5);  // T~ rows 0-31
      if (dbg && tid < 64)
        for (int i = 0; i < 64; ++i)
          p.debug[DBG_T + i * 64 + tid] =
              Tcm[tid * kTcPitch + i] + ((tid < 32 && i >= 48) ? Tcm2[tid * 20 + i - 48] : 0.f);
      signal(RDY_T, true);  // T tiles and the P tile are read by the tensor pipe
      PHASE(8)
      wait_mma(BAR_M3, par);
      PHASE(11)

      // ---- Vn^T -> bf16 A operand of (P Vn)^T; Vd^T = e^{g63 - g_t} Vn^T ->
      //      hi/lo bf16 A operands of the state update.  Lane v, tokens t in
      //      [16 cq, 16 cq + 16). ---------------------------------------------
      {
        float x[16];
        tmem_ld16(tmem + lane_base + TM_VN + 16 * cq, x);
        tmem_wait_ld();
        reg_fence(x);
        float dc[16];  // 2^(g63 - g_t) of this warp's 16 tokens (0 past the end)
        load_table16(gam + G_DEC + 16 * cq, dc);
        if constexpr (L2) {  // Vd rows / |k_t|: the state update with normalised K
          float rk[16];
          load_table16(gam + G_RK + 16 * cq, rk);
#pragma unroll
          for (int e = 0; e < 16; ++e) dc[e] *= rk[e];
        }
        if (L < kChunk) {  // partial chunk: tokens past the end contribute nothing
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (16 * cq + i >= L) x[i] = 0.f;
        }
        uint32_t wn[8], wh[8], wl[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float xv[2] = {x[2 * e], x[2 * e + 1]};
          const float2 d = mul2(xv[0], xv[1], dc[2 * e], dc[2 * e + 1]);
          wn[e] = pack_bf16x2(xv[0], xv[1]);
          const uint32_t hp = pack_bf16x2(d.x, d.y);  // round-to-nearest hi parts
          wh[e] = hp;
          const float2 lo = __fadd2_rn(d, make_float2(-bf16_lo(hp), -bf16_hi(hp)));
          wl[e] = pack_bf16x2(lo.x, lo.y);
          if (dbg) {
            p.debug[DBG_VN + (16 * cq + 2 * e) * 128 + rowv] = xv[0];
            p.debug[DBG_VN + (16 * cq + 2 * e + 1) * 128 + rowv] = xv[1];
          }
        }
        tmem_st8u(tmem + lane_base + TM_VNB + 8 * cq, wn);
        tmem_st8u(tmem + lane_base + TM_VDH + 8 * cq, wh);
        tmem_st8u(tmem + lane_base + TM_VDL + 8 * cq, wl);
        tmem_wait_st();
      }
      signal(RDY_V, false);
      if (L2 && c + 1 < nchunks) {  // next chunk's factors, in the PV wait
        wait_mma(BAR_M1, par ^ 1u);
        qk_norms(c + 1);
      }
      PHASE(12)
      if (DEBUG && dbg_cta && c == p.dbg_chunk + 2 && lane == 0) p.debug[DBG_EV + warp * 5 + 0] = float(clock64() - t_base);
      // ---- output: O[t][v] = scale (e^{gamma_t} (QS)^T[v][t] + (P Vn)^T[v][t]),
      //      lane v, tokens t in [16 cq, 16 cq + 16).  The (QS)^T half is read
      //      and scaled while the (P Vn)^T MMAs still run.  Full chunks go to the
      //      swizzled output tile (each warp store: 64 contiguous bytes of row
      //      t), stored by TMA from the issue thread; a partial chunk stores
      //      directly. ---------------------------------------------------
      {
        const bool via_tma = write_out && p.tma_out && L == kChunk;
        // lanes pair up (v even, v + 1): the even lane stores the bf16x2 words
        // of tokens 0-7 of this warp's 16, the odd lane those of tokens 8-15
        const bool odd = rowv & 1;
        const uint32_t ocol = sb + OFF_O + (rowv >> 6) * 8192 + 4 * ((rowv & 7) >> 1);
        const int och = (rowv & 63) >> 3;
        float qs[16];
        tmem_ld16(tmem + lane_base + TM_KQS + 64 + 16 * cq, qs);
        float eg[16];  // scale * 2^g_t of this warp's 16 tokens
        load_table16(gam + G_EG + 16 * cq, eg);
        if constexpr (L2) {  // Q S columns / |q_t|
          float rq[16];
          load_table16(gam + G_RQ + 16 * cq, rq);
#pragma unroll
          for (int e = 0; e < 16; ++e) eg[e] *= rq[e];
        }
        tmem_wait_ld();
        reg_fence(qs);
        float o[16];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 r = mul2(eg[i], eg[i + 1], qs[i], qs[i + 1]);
          o[i] = r.x;
          o[i + 1] = r.y;
        }
        wait_mma(BAR_PV, par);
        PHASE(13)
        if (DEBUG && dbg_cta && c == p.dbg_chunk + 2 && lane == 0) p.debug[DBG_EV + warp * 5 + 1] = float(clock64() - t_base);
        float pv[16];
        tmem_ld16(tmem + lane_base + TM_VN + 16 * cq, pv);
        tmem_wait_ld();
        reg_fence(pv);
        const int64_t tstride = static_cast<int64_t>(p.Hv_out) * kHead;
        const int64_t oelem = (t0 * p.Hv_out + h + p.head_off) * kHead + rowv;
        __nv_bfloat16* orow = p.out + oelem;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 r = __ffma2_rn(make_float2(p.scale, p.scale), make_float2(pv[i], pv[i + 1]),
                                      make_float2(o[i], o[i + 1]));
          o[i] = r.x;
          o[i + 1] = r.y;
        }
        if (via_tma) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // send what the partner keeps, receive the partner's value for ours
            const float mine = odd ? o[8 + i] : o[i];
            const float theirs = __shfl_xor_sync(0xffffffffu, odd ? o[i] : o[8 + i], 1);
            const int t = 16 * cq + (odd ? 8 : 0) + i;
            const uint32_t w = odd ? pack_bf16x2(theirs, mine) : pack_bf16x2(mine, theirs);
            sts32(ocol + t * 128 + ((och ^ (t & 7)) << 4), w);
          }
        } else if (write_out) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (16 * cq + i < L) orow[(16 * cq + i) * tstride] = __float2bfloat16_rn(o[i]);
          for (int r = 0; r < p.n_peers; ++r)
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (16 * cq + i < L) p.peer_out[r][oelem + (16 * cq + i) * tstride] = __float2bfloat16_rn(o[i]);
        }
        if (dbg)
          for (int i = 0; i < 16; ++i) {
            p.debug[DBG_QS + (16 * cq + i) * 128 + rowv] = qs[i];
            p.debug[DBG_PV + (16 * cq + i) * 128 + rowv] = pv[i];
          }
      }
      PHASE(14)
      if (DEBUG && dbg_cta && c == p.dbg_chunk + 2 && lane == 0) p.debug[DBG_EV + warp * 5 + 2] = float(clock64() - t_base);
    }
    if constexpr (DEBUG) {
      if (dbg_cta && lane == 0)
        for (int i = 0; i < kClkSlots; ++i)
          p.debug[DBG_CLK + warp * kClkSlots + i] = static_cast<float>(clk_acc[i]);
    }
#undef PHASE

    if (!aborted && write_out && p.tma_out &&
        eos - (bos + static_cast<int64_t>(nchunks - 1) * kChunk) == kChunk) {
      // output tile of the last (full) chunk
      fence_async_smem();
      named_sync(kComputeBar, kComputeThreads);
      if (tid == 0) {
        const int tl = static_cast<int>(bos + static_cast<int64_t>(nchunks - 1) * kChunk);
        const int gh = h + p.head_off;
        tma_store_3d(&tm_o, smem + OFF_O, 0, gh, tl);
        tma_store_3d(&tm_o, smem + OFF_O + 8192, 64, gh, tl);
        for (int r = 0; r < p.n_peers; ++r) {  // the same rows into every peer's buffer
          tma_store_3d(&pm.m[r], smem + OFF_O, 0, gh, tl);
          tma_store_3d(&pm.m[r], smem + OFF_O + 8192, 64, gh, tl);
        }
        bulk_commit();
        bulk_wait_all();
      }
    }

    // ---- final state -> new_state (row rowv, this warp's 32 columns) --------
    if (!aborted) {
      wait_mma(BAR_ST, static_cast<uint32_t>((nchunks - 1) & 1));
      if (!failed && ns_rows) {
        if (dbg_cta && nchunks - 1 == p.dbg_chunk) dump_state();
        // (the transpose tile is free: every warp is past the last chunk's
        // inverse, whose scratch it is)
        state_from_tmem(ns_rows + (32 * quarter) * kHead + 32 * cq, At + warp * kXposeFloats, tq_st,
                        lane);
      }
    }
  } else if (lane == 0) {
    // ======================= TMA / MMA issue thread ========================
    const uint32_t idesc_d1 = idesc_bf16(128, 64, false, false);
    const uint32_t idesc_kqs = idesc_bf16(128, 128, false, false);   // St (TMEM) x [K;Q]^T
    const uint32_t idesc_vt = idesc_bf16(128, 64, true, true);       // V^T (smem, MN) x T~^T
    const uint32_t idesc_kst = idesc_bf16(128, 64, false, true, true);  // -(KS e^g)^T (TMEM) x T~^T
    const uint32_t idesc_pv = idesc_bf16(128, 64, false, false);     // Vn^T (TMEM) x P^T
    const uint32_t idesc_st = idesc_bf16(128, 128, false, true);     // Vd^T (TMEM) x K

    const bool dbg_cta = DEBUG && p.debug && n == p.dbg_seq && h == p.dbg_head;
    long long mclk[16];
    long long mlast = 0;
    if constexpr (DEBUG) {
#pragma unroll
      for (int i = 0; i < 16; ++i) mclk[i] = 0;
      mlast = clock64();
    }
#define MPHASE(k)                             \
  if constexpr (DEBUG) {                      \
    const long long now_ = clock64();         \
    mclk[k] += now_ - mlast;                  \
    mlast = now_;                             \
  }
    int tma_issued = 0, tma_done = 0;  // chunks whose loads were issued / have landed
    auto issue_loads = [&](int cc) {
      const int s = cc & 1;
      const int tok = static_cast<int>(bos + static_cast<int64_t>(cc) * kChunk);
      uint64_t* bar = &bars[BAR_TMA0 + s];
      mbar_arrive_expect_tx(bar, v_zero ? kTmaBytes - kVStage : kTmaBytes);
      uint8_t* kq = smem + OFF_KQ + s * kKQStage;
      uint8_t* vs = smem + OFF_V + s * kVStage;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        tma_load_3d(kq + kb * 16384, &tm_k, bar, kb * 64, qh, tok);
        tma_load_3d(kq + kb * 16384 + 8192, &tm_q, bar, kb * 64, qh, tok);
        if (!v_zero) tma_load_3d(vs + kb * 8192, &tm_v, bar, kb * 64, h, tok);
      }
      tma_issued = cc + 1;
    };
    auto wait_bar = [&](int b, uint32_t parity) -> bool {
      if (!mbar_wait(&bars[b], parity, kTimeoutNs)) return false;
      tc_fence_after();
      return true;
    };
    // MMA 1 of chunk cc: [K;Q] K^T -> TM_D1 (M=128, N=64)
    auto mma1 = [&](int cc) -> bool {
      const int s = cc & 1;
      if (!wait_bar(BAR_TMA0 + s, static_cast<uint32_t>((cc >> 1) & 1))) return false;
      tma_done = cc + 1;
      MPHASE(6)
      const uint32_t kq16 = (sb + OFF_KQ + s * kKQStage) >> 4;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t d = sdesc_sw128_f(kq16 + ((ks >> 2) * 16384 + (ks & 3) * 32) / 16, 16, 1024);
        mma_bf16_ss(tmem + TM_D1, d, d, idesc_d1, ks > 0);
      }
      mma_commit(&bars[BAR_M1]);
      MPHASE(7)
      return true;
    };

    // the initial state tile (plain and ORDER instantiations), before the first chunk
    constexpr bool state_tma = STAGED;
    if (state_tma) {
      mbar_arrive_expect_tx(&bars[BAR_STATE], kHead * kHead * 4);
      const int row0 = static_cast<int>((n * p.Hv + h) * kHead);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_2d(smem + OFF_AT + c * 16384, &tm_s, &bars[BAR_STATE], 32 * c, row0);
    }
    issue_loads(0);
    if (nchunks > 1) issue_loads(1);
    bool ok = mma1(0);
    for (int c = 0; ok && c < nchunks; ++c) {
      const uint32_t par = static_cast<uint32_t>(c & 1);
      // descriptor start fields (address / 16) of this chunk's operands
      const uint32_t kq16 = (sb + OFF_KQ + (c & 1) * kKQStage) >> 4;
      const uint32_t v16 = (sb + OFF_V + (c & 1) * kVStage) >> 4;
      const uint32_t sb16 = sb >> 4;

      // (KS|QS)^T = St [K;Q]^T -> TM_KQS: A = bf16 St from TMEM (8 columns per
      // K=16 step), B = the [K;Q] rows of the stage (K-major)
      MPHASE(12)
      if (!(ok = wait_bar(RDY_S, par))) break;
      MPHASE(0)
      if (DEBUG && dbg_cta && c == p.dbg_chunk + 3) p.debug[DBG_EV + 85] = float(clock64() - t_base);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t kb = ks >> 2, kin = (ks & 3) * 32;
        mma_bf16_ts(tmem + TM_KQS, tmem + TM_SB + 8 * ks,
                    sdesc_sw128_f(kq16 + (kb * 16384 + kin) / 16, 16, 1024), idesc_kqs, ks > 0);
      }
      mma_commit(&bars[BAR_KQS]);
      // V^T Bl (the beta remainder) starts the Vn accumulator: it needs only
      // the gates, so it runs before the inverse is done
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16_ss(tmem + TM_VN, sdesc_sw128_f(v16 + ks * 128, 8192, 1024),
                    sdesc_sw128_f(sb16 + (OFF_BL + ks * 2048) / 16, 8192, 1024), idesc_vt, ks > 0);
      MPHASE(1)
      // Vn^T += V^T T~^T - (KS e^gamma)^T T~^T -> TM_VN, first over the K rows
      // 32-63 of T~ (final after level 1 of the inverse), then rows 0-31
      auto vn_mmas = [&](int ks) {
        mma_bf16_ss(tmem + TM_VN, sdesc_sw128_f(v16 + ks * 128, 8192, 1024),
                    sdesc_sw128_f(sb16 + (OFF_TB + ks * 2048) / 16, 8192, 1024), idesc_vt, 1);
        mma_bf16_ts(tmem + TM_VN, tmem + TM_KSB + 8 * ks,
                    sdesc_sw128_f(sb16 + (OFF_TB + ks * 2048) / 16, 8192, 1024), idesc_kst, 1);
      };
      if (!(ok = wait_bar(RDY_T1, par))) break;
      vn_mmas(2);
      vn_mmas(3);
      if (!(ok = wait_bar(RDY_T, par))) break;
      MPHASE(2)
      // the output tile of chunk c-1 (full: only a sequence's last chunk can be
      // partial) is complete and fenced by every compute thread before RDY_T
      if (c > 0 && p.tma_out && write_out) {
        const int tp = static_cast<int>(bos + static_cast<int64_t>(c - 1) * kChunk);
        const int gh = h + p.head_off;
        tma_store_3d(&tm_o, smem + OFF_O, 0, gh, tp);
        tma_store_3d(&tm_o, smem + OFF_O + 8192, 64, gh, tp);
        for (int r = 0; r < p.n_peers; ++r) {  // the same rows into every peer's buffer
          tma_store_3d(&pm.m[r], smem + OFF_O, 0, gh, tp);
          tma_store_3d(&pm.m[r], smem + OFF_O + 8192, 64, gh, tp);
        }
        bulk_commit();
      }
      vn_mmas(0);
      vn_mmas(1);
      mma_commit(&bars[BAR_M3]);
      MPHASE(3)
      // [K;Q]K^T of the next chunk runs while the compute warps drain Vn
      if (c + 1 < nchunks && !(ok = mma1(c + 1))) break;
      // (P Vn)^T = Vn^T P^T -> TM_VN; St += Vd_hi^T K + Vd_lo^T K
      if (!(ok = wait_bar(RDY_V, par))) break;
      MPHASE(8)
      const bool ev = DEBUG && dbg_cta && c == p.dbg_chunk + 2;
      if (ev) p.debug[DBG_EV + 80] = float(clock64() - t_base);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16_ts(tmem + TM_VN, tmem + TM_VNB + 8 * ks,
                    sdesc_sw128_f(sb16 + (OFF_P + ks * 32) / 16, 16, 1024), idesc_pv, ks > 0);
      bulk_wait_read_all();  // output tile read out before BAR_PV lets the epilogue rewrite it
      mma_commit(&bars[BAR_PV]);
      MPHASE(9)
      if (ev) p.debug[DBG_EV + 81] = float(clock64() - t_base);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16_ts(tmem + TM_ST, tmem + TM_VDH + 8 * ks, sdesc_sw128_f(kq16 + ks * 128, 16384, 1024),
                    idesc_st, 1);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_bf16_ts(tmem + TM_ST, tmem + TM_VDL + 8 * ks, sdesc_sw128_f(kq16 + ks * 128, 16384, 1024),
                    idesc_st, 1);
      mma_commit(&bars[BAR_ST]);
      MPHASE(10)
      if (ev) p.debug[DBG_EV + 82] = float(clock64() - t_base);
      // refill this chunk's stage once the state update has read K
      if (c + 2 < nchunks) {
        if (!(ok = wait_bar(BAR_ST, par))) break;
        MPHASE(11)
        if (ev) p.debug[DBG_EV + 83] = float(clock64() - t_base);
        issue_loads(c + 2);
        if (ev) p.debug[DBG_EV + 84] = float(clock64() - t_base);
      }
    }
    if constexpr (DEBUG) {
      if (dbg_cta)
        for (int i = 0; i < 16; ++i) p.debug[DBG_MCLK + i] = static_cast<float>(mclk[i]);
    }
#undef MPHASE
    // drain the tensor pipe, the output stores and any loads still in flight
    // before the CTA exits
    bulk_wait_all();
    mma_commit(&bars[BAR_END]);
    if (!mbar_wait(&bars[BAR_END], 0, kTimeoutNs)) ok = false;
    if (state_tma && !mbar_wait(&bars[BAR_STATE], 0, kTimeoutNs)) ok = false;
    for (int cc = tma_done; cc < tma_issued; ++cc)
      if (!mbar_wait(&bars[BAR_TMA0 + (cc & 1)], static_cast<uint32_t>((cc >> 1) & 1), kTimeoutNs))
        ok = false;
    failed = !ok;
  }
  if (failed) atomicOr(&g_gdn_status, kStatusPrefillTimeout);
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// A wait on an mbarrier that nothing ever arrives on, bounded by timeout_ns:
// exercises the timeout path (status word) without faulting or hanging.
__global__ void gdn_wait_probe_kernel(uint64_t timeout_ns, uint32_t* result) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, timeout_ns);
  if (threadIdx.x == 0) {
    if (!ok) atomicOr(&g_gdn_status, kStatusProbeTimeout);
    if (result) *result = ok ? 1u : 0u;
  }
}

// ---- host side ---------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// [T, heads, 128] bf16, box = 64 tokens x 1 head x 64 dims, 128-byte swizzle.
cudaError_t encode_head_map(CUtensorMap* m, const void* base, int64_t heads, int64_t T) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHead), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(T)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHead) * 2,
                           static_cast<cuuint64_t>(heads) * kHead * 2};
  cuuint32_t box[3] = {64, 1, 64};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The initial state [rows = N Hv 128][128] fp32, box 32 columns x 128 rows (one
// column quarter of a tile), 128-byte swizzle.
cudaError_t encode_state_map(CUtensorMap* m, const void* base, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHead), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHead) * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Encoding a tensor map costs about a microsecond of host time and a call needs
// four or five; a small per-thread cache of encoded maps, keyed by what the
// encoding depends on (base address, heads, T; heads = 0 marks a state map of T
// rows), skips it when a caller reuses its buffers (a serving loop, or the caching
// allocator handing back a block).
cudaError_t make_head_map(CUtensorMap* m, const void* base, int64_t heads, int64_t T) {
  struct Entry {
    const void* base;
    int64_t heads, T;
    CUtensorMap map;
  };
  constexpr int kEntries = 16;
  thread_local Entry cache[kEntries];
  thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i)
    if (cache[i].base == base && cache[i].heads == heads && cache[i].T == T) {
      *m = cache[i].map;
      return cudaSuccess;
    }
  const cudaError_t e = heads == 0 ? encode_state_map(m, base, T) : encode_head_map(m, base, heads, T);
  if (e != cudaSuccess) return e;
  cache[next] = Entry{base, heads, T, *m};
  next = (next + 1) % kEntries;
  if (used < kEntries) ++used;
  return cudaSuccess;
}

template <bool DEBUG>
cudaError_t launch_impl(const PrefillArgs& a, float* debug, int dbg_seq, int dbg_head,
                        int dbg_chunk, cudaStream_t s) {
  if ((a.jobs ? a.njobs : a.N) == 0) return cudaSuccess;
  if (a.T == 0 && !a.jobs) {  // every sequence is empty: zero final states
    return cudaMemsetAsync(a.new_state, 0,
                           static_cast<size_t>(a.N) * a.Hv * kHead * kHead * sizeof(float), s);
  }
  CUtensorMap mq, mk, mv, mo, ms;
  PeerMaps pm;
  memset(&pm, 0, sizeof(pm));
  cudaError_t e;
  const int64_t out_heads = a.out_heads > 0 ? a.out_heads : a.Hv;
  if ((e = make_head_map(&mq, a.q, a.Hq, a.T)) != cudaSuccess) return e;
  if ((e = make_head_map(&mk, a.k, a.Hq, a.T)) != cudaSuccess) return e;
  if ((e = make_head_map(&mv, a.v, a.Hv, a.T)) != cudaSuccess) return e;
  // full-chunk output rows go out by TMA store when the output allows a tensor map
  int tma_out = (reinterpret_cast<uintptr_t>(a.out) % 16 == 0) ? 1 : 0;
  for (int r = 0; r < a.n_peers; ++r)
    if (reinterpret_cast<uintptr_t>(a.peer_out[r]) % 16 != 0) tma_out = 0;
  memset(&mo, 0, sizeof(mo));
  memset(&ms, 0, sizeof(ms));
  // The initial state by TMA (the STAGED instantiation) when the sequences average
  // at most 16 chunks: it saves ~1.5 us per CTA (a 64 KiB state read as 512-byte-
  // strided rows costs a transaction per lane), but its chunk loop runs ~2.4 %
  // slower (~0.1 us per chunk), so long chains keep the plain kernel (measured:
  // one-chunk calls 11.8 -> 10.2 us, BASELINE config 2 164.8 -> 158.7 us, a 57-way
  // even split of 8192 tokens 93.2 -> 87.0 us; config 3, 256 chunks per CTA, would
  // go 1043.5 -> 1065 us).  Not for job tables, whose start states lie in two
  // buffers; TMA wants a 16-byte aligned base.
  const int64_t state_rows = a.N * a.Hv * kHead;
  const int tma_state = (!a.jobs && a.state && reinterpret_cast<uintptr_t>(a.state) % 16 == 0 &&
                         state_rows < 0x7fffffffLL && a.T <= 16 * kChunk * a.N) ? 1 : 0;
  if (tma_state && (e = make_head_map(&ms, a.state, 0, state_rows)) != cudaSuccess) return e;
  if (tma_out && (e = make_head_map(&mo, a.out, out_heads, a.T)) != cudaSuccess) return e;
  for (int r = 0; tma_out && r < a.n_peers; ++r)
    if ((e = make_head_map(&pm.m[r], a.peer_out[r], out_heads, a.T)) != cudaSuccess) return e;
  auto kernel = gdn_prefill_chunked_kernel<DEBUG, false, false, false, false>;
  const bool order = !a.jobs && a.N <= kOrderMaxSeqs && a.N * a.Hv > device_sm_count();
  // (jobs x {l2}) or (plain x {l2} x {order} x {staged})
  const int variant = a.jobs ? (a.qk_l2norm ? 1 : 0)
                             : 2 + (a.qk_l2norm ? 1 : 0) + (order ? 2 : 0) + (tma_state ? 4 : 0);
  if constexpr (!DEBUG) {
    constexpr decltype(kernel) kernels[10] = {
        gdn_prefill_chunked_kernel<false, false, true, false, false>,
        gdn_prefill_chunked_kernel<false, true, true, false, false>,
        gdn_prefill_chunked_kernel<false, false, false, false, false>,
        gdn_prefill_chunked_kernel<false, true, false, false, false>,
        gdn_prefill_chunked_kernel<false, false, false, true, false>,
        gdn_prefill_chunked_kernel<false, true, false, true, false>,
        gdn_prefill_chunked_kernel<false, false, false, false, true>,
        gdn_prefill_chunked_kernel<false, true, false, false, true>,
        gdn_prefill_chunked_kernel<false, false, false, true, true>,
        gdn_prefill_chunked_kernel<false, true, false, true, true>};
    kernel = kernels[variant];
  } else if (a.jobs || a.qk_l2norm) {
    return cudaErrorInvalidValue;  // the debug build covers the plain kernel only
  }
  // the opt-in is per device: a process may drive several GPUs
  if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), kSmemBytes)) != cudaSuccess)
    return e;
  ChunkParams p{a.state, a.A_log, a.dt_bias,
                static_cast<const __nv_bfloat16*>(a.a), static_cast<const __nv_bfloat16*>(a.b),
                a.cu_seqlens, static_cast<__nv_bfloat16*>(a.out), a.new_state, debug, a.jobs, a.scale,
                tma_out, static_cast<int>(out_heads), static_cast<int>(a.out_head_off), a.n_peers, {},
                a.T, a.N, static_cast<int>(a.Hq), static_cast<int>(a.Hv), dbg_seq, dbg_head, dbg_chunk};
  for (int r = 0; r < a.n_peers; ++r) p.peer_out[r] = static_cast<__nv_bfloat16*>(a.peer_out[r]);
  const int64_t ctas = (a.jobs ? a.njobs : a.N) * a.Hv;
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  kernel<<<static_cast<unsigned>(ctas), kThreads, kSmemBytes, s>>>(mq, mk, mv, mo, ms, pm, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_chunked(const PrefillArgs& a, cudaStream_t s) {
  return launch_impl<false>(a, nullptr, 0, 0, 0, s);
}

cudaError_t launch_prefill_chunked_debug(const PrefillArgs& a, float* debug, int dbg_seq,
                                         int dbg_head, int dbg_chunk, cudaStream_t s) {
  return launch_impl<true>(a, debug, dbg_seq, dbg_head, dbg_chunk, s);
}

int prefill_chunked_debug_floats() { return DBG_SIZE; }

cudaError_t launch_wait_probe(uint64_t timeout_ns, uint32_t* result, cudaStream_t s) {
  gdn_wait_probe_kernel<<<1, 32, 0, s>>>(timeout_ns, result);
  return cudaGetLastError();
}

cudaError_t read_status(uint32_t* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gdn_status, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  uint32_t pool = 0;  // the pooled tensor-core decode keeps its own word
  if ((e = read_pool_tc_status(&pool, clear)) != cudaSuccess) return e;
  *out |= pool;
  if (clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_gdn_status, &zero, sizeof(uint32_t));
  }
  return e;
}

}  // namespace gdn
