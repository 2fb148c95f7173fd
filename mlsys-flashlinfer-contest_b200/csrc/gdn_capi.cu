// C ABI of the gdn_b200 library: validation, dispatch and error reporting.
// Declarations and the contract of each entry point: include/gdn_b200.h.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "../../include/gdn_b200.h"
#include "gdn_internal.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return GDN_OK;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s failed: %s", what, cudaGetErrorString(e));
  return ok();
}

bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// [p, p+bytes) and [q, q+bytes) overlap without being identical
bool partial_overlap(const void* p, const void* q, size_t bytes) {
  if (p == nullptr || q == nullptr || p == q) return false;
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return a < b + bytes && b < a + bytes;
}

int check_heads(int64_t Hq, int64_t Hk, int64_t Hv, int64_t D) {
  if (D != gdn::kHead) return fail(GDN_ERR_VALUE, "head_size must be 128 (got %lld)", (long long)D);
  if (Hq <= 0 || Hk <= 0) return fail(GDN_ERR_VALUE, "head counts must be positive");
  if (Hk != Hq)
    return fail(GDN_ERR_VALUE, "num_k_heads (%lld) must equal num_q_heads (%lld)", (long long)Hk,
                (long long)Hq);
  if (Hv < Hq || Hv % Hq != 0)
    return fail(GDN_ERR_VALUE, "num_v_heads (%lld) must be a multiple of num_q_heads (%lld)",
                (long long)Hv, (long long)Hq);
  return GDN_OK;
}

int64_t upper_bound_chunks(int64_t T, int64_t N) {
  if (T <= 0 || N <= 0) return 0;
  if (T < N) return T;
  return N + (T - N) / gdn::kChunk;
}

}  // namespace

extern "C" {

int gdn_abi_version(void) { return GDN_ABI_VERSION; }

const char* gdn_last_error(void) { return g_err; }

int64_t gdn_chunk_upper_bound(int64_t T, int64_t N) { return upper_bound_chunks(T, N); }

int gdn_decode(const void* q, const void* k, const void* v, const float* state, const float* A_log,
               const void* a, const float* dt_bias, const void* b, float scale, void* output,
               float* new_state, int64_t B, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D,
               void* stream) {
  if (int e = check_heads(Hq, Hk, Hv, D)) return e;
  if (B < 0) return fail(GDN_ERR_VALUE, "batch_size must be non-negative");
  if (B == 0) return ok();
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !output || !new_state)
    return fail(GDN_ERR_VALUE, "null pointer argument");
  if (!aligned(q, 8) || !aligned(k, 8))
    return fail(GDN_ERR_VALUE, "q and k must be 8-byte aligned");
  if (!aligned(new_state, 16) || (state && !aligned(state, 16)))
    return fail(GDN_ERR_VALUE, "state and new_state must be 16-byte aligned");
  const size_t state_bytes = static_cast<size_t>(B) * Hv * gdn::kHead * gdn::kHead * 4;
  if (partial_overlap(state, new_state, state_bytes))
    return fail(GDN_ERR_VALUE, "new_state overlaps state without being the same buffer");
  gdn::DecodeArgs p{q, k, v, state, A_log, a, dt_bias, b, scale == 0.0f ? 0.08838834764831845f : scale,
                    output, new_state, B, Hq, Hv};
  return cuda_status(gdn::launch_decode(p, 0, static_cast<cudaStream_t>(stream)), "gdn_decode launch");
}

int gdn_decode_pool(const void* q, const void* k, const void* v, const float* A_log, const void* a,
                    const float* dt_bias, const void* b, float scale, void* pool, int state_dtype,
                    int64_t pool_size, const int32_t* in_slots, const int32_t* out_slots,
                    void* intermediate, int flags, void* output, int64_t B, int64_t T, int64_t Hq,
                    int64_t Hk, int64_t Hv, int64_t D, void* stream) {
  if (int e = check_heads(Hq, Hk, Hv, D)) return e;
  if (B < 0) return fail(GDN_ERR_VALUE, "batch_size must be non-negative");
  if (T < 1) return fail(GDN_ERR_VALUE, "seq_len must be at least 1");
  if (pool_size < 0) return fail(GDN_ERR_VALUE, "pool_size must be non-negative");
  if (pool_size > INT32_MAX) return fail(GDN_ERR_VALUE, "pool_size must fit int32 slot indices");
  if (state_dtype != GDN_STATE_F32 && state_dtype != GDN_STATE_BF16)
    return fail(GDN_ERR_TYPE, "state_dtype must be GDN_STATE_F32 or GDN_STATE_BF16");
  if (flags & ~(GDN_POOL_QK_L2NORM | GDN_POOL_NO_STATE_UPDATE))
    return fail(GDN_ERR_VALUE, "unknown flags");
  if (B == 0) return ok();
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !output || !in_slots)
    return fail(GDN_ERR_VALUE, "null pointer argument");
  if (pool_size > 0 && !pool) return fail(GDN_ERR_VALUE, "null pointer argument");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(pool, 16) ||
      !aligned(intermediate, 16))
    return fail(GDN_ERR_VALUE, "q, k, v, state_pool and intermediate must be 16-byte aligned");
  if (!aligned(in_slots, 4) || !aligned(out_slots, 4))
    return fail(GDN_ERR_VALUE, "slot arrays must be 4-byte aligned");
  gdn::DecodePoolArgs p{q, k, v, A_log, a, dt_bias, b, scale == 0.0f ? 0.08838834764831845f : scale,
                        pool, in_slots, out_slots, intermediate, output, B, T, Hq, Hv, pool_size,
                        state_dtype == GDN_STATE_BF16, (flags & GDN_POOL_QK_L2NORM) != 0,
                        (flags & GDN_POOL_NO_STATE_UPDATE) != 0};
  return cuda_status(gdn::launch_decode_pool(p, static_cast<cudaStream_t>(stream)),
                     "gdn_decode_pool launch");
}

static int check_prefill(const void* q, const void* k, const void* v, const float* state,
                         const float* A_log, const void* a, const float* dt_bias, const void* b,
                         const int64_t* cu, void* out, float* new_state, int64_t T, int64_t N,
                         int64_t Hq, int64_t Hk, int64_t Hv, int64_t D) {
  if (int e = check_heads(Hq, Hk, Hv, D)) return e;
  if (N <= 0) return fail(GDN_ERR_VALUE, "must have at least one sequence");
  if (T < 0) return fail(GDN_ERR_VALUE, "total_seq_len must be non-negative");
  if (!cu || !A_log || !dt_bias || !new_state) return fail(GDN_ERR_VALUE, "null pointer argument");
  if (T > 0 && (!q || !k || !v || !a || !b || !out)) return fail(GDN_ERR_VALUE, "null pointer argument");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16))
    return fail(GDN_ERR_VALUE, "q, k and v must be 16-byte aligned");
  if (!aligned(new_state, 16) || (state && !aligned(state, 16)))
    return fail(GDN_ERR_VALUE, "state and new_state must be 16-byte aligned");
  if (!aligned(cu, 8)) return fail(GDN_ERR_VALUE, "cu_seqlens must be 8-byte aligned");
  const size_t state_bytes = static_cast<size_t>(N) * Hv * gdn::kHead * gdn::kHead * 4;
  if (partial_overlap(state, new_state, state_bytes))
    return fail(GDN_ERR_VALUE, "new_state overlaps state without being the same buffer");
  return GDN_OK;
}

int gdn_prefill_recurrent(const void* q, const void* k, const void* v, const float* state,
                          const float* A_log, const void* a, const float* dt_bias, const void* b,
                          const int64_t* cu_seqlens, float scale, void* output, float* new_state,
                          int64_t T, int64_t N, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D,
                          void* stream) {
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv};
  return cuda_status(gdn::launch_prefill_recurrent(p, static_cast<cudaStream_t>(stream)),
                     "gdn_prefill_recurrent launch");
}

// Chooses the token-recurrent kernel for tiny inputs and the fused chunked
// kernel otherwise.  The reference dispatches on the same two sizes
// (gdn_prefill/solution/python/gdn_prefill_mix.py:29: N <= 2 and T <= 30 N);
// the bounds here come from timing both kernels on a B200 over N = 1..32
// sequences of 8..512 tokens (Hv = 8 and 32): the recurrent kernel walks one
// token at a time (~0.3 us each) while the chunked kernel's floor is one chunk
// (~14.5 us per call, launch included).  Recurrent wins for sequences of up to
// ~32 tokens when there are at most 16 (sequence, head) pairs, up to 16 tokens
// at up to 64 pairs, and up to 8 tokens at any count.  The last bound also caps
// T, because only the mean length is known on the host: one long sequence among
// many short ones walks all its tokens.
static bool use_recurrent(int64_t T, int64_t N, int64_t Hv) {
  return (T <= 32 * N && N * Hv <= 16) || (T <= 16 * N && N * Hv <= 64) ||
         (T <= 8 * N && T <= 256);
}

// Upper bound on the piece count of the sequence-parallel prefill (1: one chain
// per (sequence, head)).  The job builder picks each sequence's count under it
// from the lengths on the device (the shortest longest chain whose passes fit the
// SMs: pass 1 within one to three waves of the SMs its piece-0 jobs leave free,
// pass 2 within one wave), so the host only rules out calls that cannot gain:
// more (sequence, head) pairs than half the SMs (then not even equal sequences
// could all be cut in 3 with pass 2 in one wave), or fewer chunks in all than
// the shortest sequence the builder would cut (prefill_min_cut_chunks); the
// bound is the largest G <= kMaxAutoSegments with N Hv (G - 1) <= 2 SMs and
// T >= 4 G chunks.
static int sm_count() { return gdn::device_sm_count(); }
constexpr int kMaxAutoSegments = 16;

static int choose_segments(int64_t T, int64_t N, int64_t Hv) {
  if (N <= 0 || Hv <= 0 || 2 * N * Hv > sm_count()) return 1;
  const int64_t chunks = T / gdn::kChunk;
  // no sequence can be long enough for the builder to accept a cut: the
  // segmented form would only add its launches
  if ((T + gdn::kChunk - 1) / gdn::kChunk < gdn::prefill_min_cut_chunks()) return 1;
  int best = 1;
  for (int G = 3; G <= kMaxAutoSegments; ++G)
    if (N * Hv * (G - 1) <= 2 * sm_count() && chunks >= 4 * G) best = G;
  return best;
}

int gdn_prefill_segments(int64_t T, int64_t N, int64_t Hv) {
  return use_recurrent(T, N, Hv) ? 1 : choose_segments(T, N, Hv);
}

// segments 0: the automatic form (sized for the largest bound)
size_t gdn_prefill_segmented_workspace_bytes(int64_t N, int64_t Hv, int segments) {
  if (segments == 0) return gdn::prefill_segments_bytes(N, Hv, kMaxAutoSegments, true, sm_count());
  return gdn::prefill_segments_bytes(N, Hv, segments, false, sm_count());
}

size_t gdn_prefill_workspace_bytes(int64_t T, int64_t N, int64_t Hq, int64_t Hv) {
  (void)Hq;
  const int G = gdn_prefill_segments(T, N, Hv);
  return G > 1 ? gdn::prefill_segments_bytes(N, Hv, G, true, sm_count()) : 0;
}

int gdn_prefill_chunked(const void* q, const void* k, const void* v, const float* state,
                        const float* A_log, const void* a, const float* dt_bias, const void* b,
                        const int64_t* cu_seqlens, float scale, void* output, float* new_state,
                        int64_t T, int64_t N, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D,
                        void* stream) {
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (T > 0x7fffffffLL - 64) return fail(GDN_ERR_VALUE, "total_seq_len too large");
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv};
  return cuda_status(gdn::launch_prefill_chunked(p, static_cast<cudaStream_t>(stream)),
                     "gdn_prefill_chunked launch");
}

int gdn_prefill(const void* q, const void* k, const void* v, const float* state, const float* A_log,
                const void* a, const float* dt_bias, const void* b, const int64_t* cu_seqlens,
                float scale, void* output, float* new_state, int64_t T, int64_t N, int64_t Hq,
                int64_t Hk, int64_t Hv, int64_t D, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (use_recurrent(T, N, Hv))
    return gdn_prefill_recurrent(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                                 new_state, T, N, Hq, Hk, Hv, D, stream);
  const int G = choose_segments(T, N, Hv);
  if (G > 1 && workspace && workspace_bytes >= gdn::prefill_segments_bytes(N, Hv, G, true, sm_count()))
    return gdn_prefill_segmented(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                                 new_state, T, N, Hq, Hk, Hv, D, 0, 0, workspace, workspace_bytes,
                                 stream);
  return gdn_prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                             new_state, T, N, Hq, Hk, Hv, D, stream);
}

// Checks shared by the segmented entries; segments 0 = automatic (an upper bound
// for the device's per-sequence choice).
static int segmented_setup(int64_t T, int64_t N, int64_t Hv, int* segments, bool* adaptive,
                           void* workspace, size_t workspace_bytes) {
  if (*segments < 0 || *segments > 64) return fail(GDN_ERR_VALUE, "segments must be in [0, 64]");
  *adaptive = *segments == 0;
  if (*adaptive) *segments = choose_segments(T, N, Hv);
  const size_t need = gdn::prefill_segments_bytes(N, Hv, *segments, *adaptive, sm_count());
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(GDN_ERR_VALUE, "workspace needs %zu bytes", need);
  if (!aligned(workspace, 256)) return fail(GDN_ERR_VALUE, "workspace must be 256-byte aligned");
  return GDN_OK;
}

int gdn_prefill_segmented(const void* q, const void* k, const void* v, const float* state,
                          const float* A_log, const void* a, const float* dt_bias, const void* b,
                          const int64_t* cu_seqlens, float scale, void* output, float* new_state,
                          int64_t T, int64_t N, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D,
                          int flags, int segments, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (flags & ~GDN_PREFILL_QK_L2NORM) return fail(GDN_ERR_VALUE, "unknown flags");
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (T > 0x7fffffffLL - 64) return fail(GDN_ERR_VALUE, "total_seq_len too large");
  bool adaptive = false;
  if (int e = segmented_setup(T, N, Hv, &segments, &adaptive, workspace, workspace_bytes)) return e;
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv,
                     (flags & GDN_PREFILL_QK_L2NORM) != 0};
  return cuda_status(gdn::launch_prefill_segmented(p, segments, adaptive, sm_count(), workspace,
                                                   workspace_bytes, static_cast<cudaStream_t>(stream)),
                     "gdn_prefill_segmented launch");
}

int gdn_prefill_ex(const void* q, const void* k, const void* v, const float* state,
                   const float* A_log, const void* a, const float* dt_bias, const void* b,
                   const int64_t* cu_seqlens, float scale, void* output, float* new_state, int64_t T,
                   int64_t N, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D, int flags, int path,
                   void* stream) {
  if (flags & ~GDN_PREFILL_QK_L2NORM) return fail(GDN_ERR_VALUE, "unknown flags");
  if (path < GDN_PREFILL_PATH_AUTO || path > GDN_PREFILL_PATH_CHUNKED)
    return fail(GDN_ERR_VALUE, "unknown path");
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (T > 0x7fffffffLL - 64) return fail(GDN_ERR_VALUE, "total_seq_len too large");
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv,
                     (flags & GDN_PREFILL_QK_L2NORM) != 0};
  const bool recurrent =
      path == GDN_PREFILL_PATH_RECURRENT || (path == GDN_PREFILL_PATH_AUTO && use_recurrent(T, N, Hv));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  return recurrent ? cuda_status(gdn::launch_prefill_recurrent(p, st), "gdn_prefill_recurrent launch")
                   : cuda_status(gdn::launch_prefill_chunked(p, st), "gdn_prefill_chunked launch");
}

// No-allocation form of gdn_prefill_segmented: the scratch is the library's own
// device array (gdn::kNoAllocScratchBytes per GPU), whose address on the current
// device is looked up on the first call on that device.
int gdn_prefill_segmented_noalloc(const void* q, const void* k, const void* v, const float* state,
                                  const float* A_log, const void* a, const float* dt_bias,
                                  const void* b, const int64_t* cu_seqlens, float scale,
                                  void* output, float* new_state, int64_t T, int64_t N, int64_t Hq,
                                  int64_t Hk, int64_t Hv, int64_t D, int flags, int segments,
                                  void* stream) {
  static_assert(GDN_NOALLOC_SCRATCH_BYTES == gdn::kNoAllocScratchBytes, "scratch size");
  if (flags & ~GDN_PREFILL_QK_L2NORM) return fail(GDN_ERR_VALUE, "unknown flags");
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (T > 0x7fffffffLL - 64) return fail(GDN_ERR_VALUE, "total_seq_len too large");
  if (segments < 0 || segments > 64) return fail(GDN_ERR_VALUE, "segments must be in [0, 64]");
  const bool adaptive = segments == 0;
  if (adaptive) segments = choose_segments(T, N, Hv);
  const size_t need = gdn::prefill_segments_bytes(N, Hv, segments, adaptive, sm_count());
  if (need > gdn::kNoAllocScratchBytes)
    return fail(GDN_ERR_VALUE,
                "%lld sequences x %lld heads in %d pieces need %zu bytes of scratch; the "
                "no-allocation entry holds %zu (use gdn_prefill_segmented with a workspace)",
                static_cast<long long>(N), static_cast<long long>(Hv), segments, need,
                gdn::kNoAllocScratchBytes);
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv,
                     (flags & GDN_PREFILL_QK_L2NORM) != 0};
  return cuda_status(gdn::launch_prefill_segmented_noalloc(p, segments, adaptive, sm_count(),
                                                           static_cast<cudaStream_t>(stream)),
                     "gdn_prefill_segmented_noalloc launch");
}

int gdn_prefill_chunked_peers(const void* q, const void* k, const void* v, const float* state,
                              const float* A_log, const void* a, const float* dt_bias, const void* b,
                              const int64_t* cu_seqlens, float scale, void* output, float* new_state,
                              int64_t T, int64_t N, int64_t Hq, int64_t Hk, int64_t Hv, int64_t D,
                              int64_t Hv_out, int64_t head_offset, void* const* peer_outputs,
                              int num_peers, int segments, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (T > 0x7fffffffLL - 64) return fail(GDN_ERR_VALUE, "total_seq_len too large");
  if (num_peers < 0 || num_peers > gdn::kMaxPeers)
    return fail(GDN_ERR_VALUE, "num_peers must be in [0, %d]", gdn::kMaxPeers);
  if (num_peers > 0 && !peer_outputs) return fail(GDN_ERR_VALUE, "null pointer argument");
  if (head_offset < 0 || Hv_out < Hv || head_offset + Hv > Hv_out || Hv_out > 0x7fffffffLL)
    return fail(GDN_ERR_VALUE, "heads [head_offset, head_offset + num_v_heads) must lie in the output");
  if (!aligned(output, 16)) return fail(GDN_ERR_VALUE, "output must be 16-byte aligned");
  for (int r = 0; r < num_peers; ++r)
    if (!peer_outputs[r] || !aligned(peer_outputs[r], 16))
      return fail(GDN_ERR_VALUE, "peer output %d is null or not 16-byte aligned", r);
  bool adaptive = false;
  if (int e = segmented_setup(T, N, Hv, &segments, &adaptive, workspace, workspace_bytes)) return e;
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv};
  p.out_heads = Hv_out;
  p.out_head_off = head_offset;
  p.n_peers = num_peers;
  p.peer_out = peer_outputs;
  return cuda_status(gdn::launch_prefill_segmented(p, segments, adaptive, sm_count(), workspace,
                                                   workspace_bytes, static_cast<cudaStream_t>(stream)),
                     "gdn_prefill_chunked_peers launch");
}

int gdn_prefill_chunked_debug(const void* q, const void* k, const void* v, const float* state,
                              const float* A_log, const void* a, const float* dt_bias,
                              const void* b, const int64_t* cu_seqlens, float scale, void* output,
                              float* new_state, int64_t T, int64_t N, int64_t Hq, int64_t Hk,
                              int64_t Hv, int64_t D, float* debug, int64_t debug_floats,
                              int64_t dbg_seq, int64_t dbg_head, int64_t dbg_chunk, void* stream) {
  if (int e = check_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, T,
                            N, Hq, Hk, Hv, D))
    return e;
  if (!debug || debug_floats < gdn::prefill_chunked_debug_floats())
    return fail(GDN_ERR_VALUE, "debug buffer needs %d floats", gdn::prefill_chunked_debug_floats());
  gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                     scale == 0.0f ? 0.08838834764831845f : scale, output, new_state, T, N, Hq, Hv};
  return cuda_status(
      gdn::launch_prefill_chunked_debug(p, debug, static_cast<int>(dbg_seq),
                                        static_cast<int>(dbg_head), static_cast<int>(dbg_chunk),
                                        static_cast<cudaStream_t>(stream)),
      "gdn_prefill_chunked_debug launch");
}

int64_t gdn_prefill_chunked_debug_floats(void) { return gdn::prefill_chunked_debug_floats(); }

int gdn_read_status(uint32_t* status, int clear) {
  if (!status) return fail(GDN_ERR_VALUE, "null pointer argument");
  return cuda_status(gdn::read_status(status, clear != 0), "gdn_read_status");
}

int gdn_wait_probe(uint64_t timeout_ns, uint32_t* result, void* stream) {
  if (timeout_ns > 5000000000ull) return fail(GDN_ERR_VALUE, "timeout_ns must be <= 5 s");
  return cuda_status(gdn::launch_wait_probe(timeout_ns, result, static_cast<cudaStream_t>(stream)),
                     "gdn_wait_probe launch");
}

int gdn_prep_meta(const int64_t* cu_seqlens, int64_t N, int32_t* chunk_offsets,
                  int32_t* chunk_indices, int64_t max_chunks, void* stream) {
  if (N < 0) return fail(GDN_ERR_VALUE, "num_seqs must be non-negative");
  if (!cu_seqlens || !chunk_offsets || (max_chunks > 0 && !chunk_indices))
    return fail(GDN_ERR_VALUE, "null pointer argument");
  if (!aligned(chunk_indices, 8)) return fail(GDN_ERR_VALUE, "chunk_indices must be 8-byte aligned");
  return cuda_status(gdn::launch_prep_meta(cu_seqlens, N, chunk_offsets, chunk_indices, max_chunks,
                                           static_cast<cudaStream_t>(stream)),
                     "gdn_prep_meta launch");
}

}  // extern "C"
