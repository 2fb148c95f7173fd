// Internal launch interfaces between the C-ABI layer (gdn_capi.cu) and the
// kernel translation units.  Not part of the public header.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gdn {

#ifndef GDN_CONSTANTS_DEFINED
#define GDN_CONSTANTS_DEFINED
constexpr int kHead = 128;   // head_size (K = V = 128, fixed by the definitions)
constexpr int kChunk = 64;   // chunk length of the chunked prefill
#endif

// SM count of the current device (cached per device).
int device_sm_count();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `func` on the current
// device, once per (device, function); a no-op up to the 48 KiB default.
cudaError_t set_max_dynamic_smem(const void* func, int bytes);

struct DecodeArgs {
  const void* q;        // [B,1,Hq,128] bf16
  const void* k;        // [B,1,Hk,128] bf16 (Hk == Hq)
  const void* v;        // [B,1,Hv,128] bf16
  const float* state;   // [B,Hv,128,128] fp32 k-last, or nullptr (zero state)
  const float* A_log;   // [Hv]
  const void* a;        // [B,1,Hv] bf16
  const float* dt_bias; // [Hv]
  const void* b;        // [B,1,Hv] bf16
  float scale;          // already resolved (0 -> 1/sqrt(128))
  void* out;            // [B,1,Hv,128] bf16
  float* new_state;     // [B,Hv,128,128] fp32 (may equal state)
  int64_t B, Hq, Hv;
};

// rows_per_cta: 0 = choose from the problem size, else 32, 64 or 128.
cudaError_t launch_decode(const DecodeArgs& a, int rows_per_cta, cudaStream_t s);

struct DecodePoolArgs {
  const void* q;           // [B,T,Hq,128] bf16
  const void* k;           // [B,T,Hk,128] bf16
  const void* v;           // [B,T,Hv,128] bf16
  const float* A_log;      // [Hv]
  const void* a;           // [B,T,Hv] bf16
  const float* dt_bias;    // [Hv]
  const void* b;           // [B,T,Hv] bf16
  float scale;             // already resolved
  void* pool;              // [pool_size,Hv,128,128] fp32 or bf16 (state_bf16)
  const int32_t* in_slots;   // [B] device
  const int32_t* out_slots;  // [B] device, or nullptr (= in_slots)
  void* intermediate;      // [B,T,Hv,128,128] in the pool's dtype, or nullptr
  void* out;               // [B,T,Hv,128] bf16
  int64_t B, T, Hq, Hv, pool_size;
  bool state_bf16, qk_l2norm, no_state_update;
};

cudaError_t launch_decode_pool(const DecodePoolArgs& a, cudaStream_t s);
// Tensor-core multi-token form for bf16 pools (3 <= T <= 16, no per-token state
// cache): the 2T dot products of every state row with the tokens' k and q in one
// tcgen05 MMA, then a closed-form triangular solve and one rank-T state update;
// persistent, warp-specialised (TMA loader, MMA issuer, gates, tables, solve and
// update warps).
bool decode_pool_tc_supported(const DecodePoolArgs& a);
cudaError_t launch_decode_pool_tc(const DecodePoolArgs& a, cudaStream_t s);
cudaError_t read_pool_tc_status(uint32_t* out, bool clear);

struct PrefillArgs {
  const void* q;           // [T,Hq,128] bf16
  const void* k;           // [T,Hk,128] bf16
  const void* v;           // [T,Hv,128] bf16
  const float* state;      // [N,Hv,128,128] fp32 or nullptr
  const float* A_log;      // [Hv]
  const void* a;           // [T,Hv] bf16
  const float* dt_bias;    // [Hv]
  const void* b;           // [T,Hv] bf16
  const int64_t* cu_seqlens;  // [N+1] int64, device
  float scale;
  void* out;               // [T,Hv,128] bf16
  float* new_state;        // [N,Hv,128,128] fp32
  int64_t T, N, Hq, Hv;
  bool qk_l2norm = false;  // L2-normalise q and k per head: x / sqrt(sum x^2 + 1e-6)
  // output routing (chunked kernel): `out` holds out_heads heads (0 = Hv) and this
  // call's heads land at [out_head_off, out_head_off + Hv); each of the n_peers
  // peer-mapped buffers of the same shape gets the same rows (the all-gather of a
  // head-sharded call, done by the kernel's own stores over NVLink)
  int64_t out_heads = 0, out_head_off = 0;
  int n_peers = 0;
  void* const* peer_out = nullptr;
  // chunked kernel only: a job table in device memory (one job per group of Hv
  // CTAs) replaces cu_seqlens / state / new_state when set
  const struct SegJob* jobs = nullptr;
  int64_t njobs = 0;
};

// One job of the segmented prefill: the tokens [bos, eos) of one sequence
// segment for all Hv heads, from state_in ([Hv,128,128] fp32; nullptr = zero;
// ignored with kJobIdentity) to state_out ([Hv,128,128]; nullptr = not stored).
enum : uint32_t {
  kJobIdentity = 1u,  // initial state = identity (the segment's transition matrix)
  kJobNoV = 2u,       // v = 0
  kJobNoOut = 4u,     // outputs not written
};
struct SegJob {
  int64_t bos, eos;
  const float* state_in;
  float* state_out;
  uint32_t flags, pad;
};
constexpr int kMaxPeers = 7;

cudaError_t launch_prefill_recurrent(const PrefillArgs& a, cudaStream_t s);
// Segmented (sequence-parallel) prefill: sequences are cut into pieces at chunk
// boundaries; pass 1 runs piece 0 from the initial state and, for the middle
// pieces, their final state from zero (F) and their transition matrix (P, the
// final state from the identity with v = 0); the start states of pieces 2..
// follow from S_{g+1} = S_g P_g + F_g in fp32; pass 2 runs pieces 1.. from
// their start states.  adaptive: `segments` is an upper bound and the device
// picks each sequence's count (pass 1 within `sms` CTAs); else every sequence of
// at least 2 segments chunks is cut into `segments`.
size_t prefill_segments_bytes(int64_t N, int64_t Hv, int segments, bool adaptive, int sms);
// The fewest chunks a sequence needs before the automatic form can cut it.
int prefill_min_cut_chunks();
cudaError_t launch_prefill_segmented(const PrefillArgs& a, int segments, bool adaptive, int sms,
                                     void* workspace, size_t workspace_bytes, cudaStream_t s);
// The same with the workspace in a file-scope device array of kNoAllocScratchBytes
// (the no-allocation entry); the caller checks prefill_segments_bytes against it.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
cudaError_t launch_prefill_segmented_noalloc(const PrefillArgs& a, int segments, bool adaptive,
                                             int sms, cudaStream_t s);

// fused chunked (C=64) prefill on tcgen05 (a job table in PrefillArgs: the
// segmented form's passes)
cudaError_t launch_prefill_chunked(const PrefillArgs& a, cudaStream_t s);
// same kernel, dumping one chunk's intermediates (gamma, beta, A, P, T, U, W,
// Vn, QS, PV, St) of (dbg_seq, dbg_head, dbg_chunk) into `debug`
cudaError_t launch_prefill_chunked_debug(const PrefillArgs& a, float* debug, int dbg_seq,
                                         int dbg_head, int dbg_chunk, cudaStream_t s);
int prefill_chunked_debug_floats();

// bounded wait on an mbarrier nothing arrives on (timeout path test)
cudaError_t launch_wait_probe(uint64_t timeout_ns, uint32_t* result, cudaStream_t s);
// device status word (bit flags of kernels that gave up on a wait)
cudaError_t read_status(uint32_t* out, bool clear);

// chunk metadata: offsets [N+1] int32, indices [max_chunks,2] int32
cudaError_t launch_prep_meta(const int64_t* cu_seqlens, int64_t N, int32_t* chunk_offsets,
                             int32_t* chunk_indices, int64_t max_chunks, cudaStream_t s);

}  // namespace gdn
