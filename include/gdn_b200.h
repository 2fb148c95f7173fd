/*
 * gdn_b200 -- C ABI of the B200 (sm_100a) Gated DeltaNet decode / prefill kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle
 * (a cudaStream_t passed as void*; NULL = the legacy default stream).  Nothing
 * is allocated, freed or synchronised inside a call: the caller owns every
 * buffer, including the prefill workspace, and the call returns as soon as the
 * kernels are enqueued.  Tensors are dense and contiguous in the layouts of the
 * reference definitions (definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md,
 * definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md):
 *
 *   bf16 tensors are passed as `const void *` holding IEEE bfloat16 values;
 *   head_size must be 128; num_k_heads == num_q_heads;
 *   num_v_heads % num_q_heads == 0 (GVA: v-head h reads q/k head h / (Hv/Hq));
 *   the recurrent state is fp32 in the k-last layout [.., Hv, V=128, K=128].
 *
 * Return value: GDN_OK, or an error code whose message is available from
 * gdn_last_error() (thread-local).  The codes map onto the exception types of
 * the reference's TVM-FFI checks (gdn_decode/solution/python/gdn_decode_utils.h:16-122):
 * GDN_ERR_VALUE -> ValueError, GDN_ERR_TYPE -> TypeError, GDN_ERR_CUDA -> RuntimeError.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 1

enum gdn_status {
  GDN_OK = 0,
  GDN_ERR_VALUE = 1,   /* bad size, count, pointer or alignment */
  GDN_ERR_TYPE = 2,    /* reserved for dtype errors raised by bindings */
  GDN_ERR_CUDA = 3,    /* a CUDA launch or runtime call failed */
};

/* ABI version of the loaded library (GDN_ABI_VERSION). */
int gdn_abi_version(void);

/* Message of the last failed call on this thread ("" after a success). */
const char *gdn_last_error(void);

/*
 * Decode one token per sequence.
 * Replaces the reference's decode FFI entry points
 *   gdn_decode_small_batch  (gdn_decode/solution/python/gdn_decode_small_batch.cu:194-232)
 *   large_batch run         (gdn_decode/solution/python/gdn_decode_kernel_large_batch.py:343-406)
 * behind the solution entry gdn_decode/solution/python/gdn_decode_final.py:23-36.
 *
 *   q, k      [B, 1, Hq, 128] bf16         v        [B, 1, Hv, 128] bf16
 *   state     [B, Hv, 128, 128] fp32 or NULL (= zero initial state)
 *   A_log, dt_bias [Hv] fp32               a, b     [B, 1, Hv] bf16
 *   scale     0 selects 1/sqrt(128)
 *   output    [B, 1, Hv, 128] bf16         new_state [B, Hv, 128, 128] fp32
 * new_state may equal state (in-place update); any other overlap is rejected.
 * q, k need 8-byte alignment, state and new_state 16-byte alignment.
 */
int gdn_decode(const void *q, const void *k, const void *v, const float *state,
               const float *A_log, const void *a, const float *dt_bias, const void *b,
               float scale, void *output, float *new_state, int64_t batch_size,
               int64_t num_q_heads, int64_t num_k_heads, int64_t num_v_heads,
               int64_t head_size, void *stream);

/* Storage type of a pooled state (gdn_decode_pool). */
enum gdn_state_dtype { GDN_STATE_F32 = 0, GDN_STATE_BF16 = 1 };
/* gdn_decode_pool flags */
#define GDN_POOL_QK_L2NORM 1        /* L2-normalise q and k per head: x / sqrt(sum x^2 + 1e-6) */
#define GDN_POOL_NO_STATE_UPDATE 2  /* leave the pool untouched (outputs / cache only) */

/*
 * Pooled multi-token decode: the serving form of gdn_decode.  No reference
 * counterpart: the reference workspace decodes one token per sequence with a
 * dense fp32 state batch (gdn_decode_final.py:23-36); this entry is the adjacent
 * "next" variant (bf16 state, multi-token, in-kernel q/k L2 norm) that installed
 * FlashInfer ships as gdn_decode_bf16_state / gdn_decode_mtp.
 *
 *   q, k      [B, T, Hq, 128] bf16        v        [B, T, Hv, 128] bf16
 *   A_log, dt_bias [Hv] fp32              a, b     [B, T, Hv] bf16
 *   state_pool [pool_size, Hv, 128, 128] in state_dtype (k-last)
 *   in_slots  [B] int32 device: pool slot each sequence starts from; a negative
 *             or out-of-range slot means a zero initial state
 *   out_slots [B] int32 device or NULL (= in_slots): slot each final state is
 *             written to; negative or out-of-range: not written
 *   intermediate NULL or [B, T, Hv, 128, 128] in state_dtype: state after each token
 *   output    [B, T, Hv, 128] bf16
 * Tokens of a sequence are applied in order t = 0..T-1 (T >= 1), the state kept
 * in fp32 registers between them and rounded to state_dtype once per store.  The
 * pool is updated in place; two sequences writing the same slot, or one reading a
 * slot another writes, race.  All buffers need 16-byte alignment.
 */
int gdn_decode_pool(const void *q, const void *k, const void *v, const float *A_log,
                    const void *a, const float *dt_bias, const void *b, float scale,
                    void *state_pool, int state_dtype, int64_t pool_size,
                    const int32_t *in_slots, const int32_t *out_slots, void *intermediate,
                    int flags, void *output, int64_t batch_size, int64_t seq_len,
                    int64_t num_q_heads, int64_t num_k_heads, int64_t num_v_heads,
                    int64_t head_size, void *stream);

/*
 * Prefill packed variable-length sequences.
 * Replaces the solution entry gdn_prefill/solution/python/gdn_prefill_mix.py:13-38
 * and the FFI calls it makes: gdn_prefill_recurrent_v1 (cuda_recurrent_v1.cu:232-277)
 * for tiny inputs, else the chunked pipeline of chunk_v12.py:36-116 (prep_meta_v2,
 * kkt_inv_uw_v1, h_v2b, o_v1).
 *
 *   q, k      [T, Hq, 128] bf16            v        [T, Hv, 128] bf16
 *   state     [N, Hv, 128, 128] fp32 or NULL (= zero initial states)
 *   a, b      [T, Hv] bf16                 cu_seqlens [N+1] int64, device memory,
 *                                          non-decreasing, cu_seqlens[N] == T
 *   output    [T, Hv, 128] bf16            new_state [N, Hv, 128, 128] fp32
 *   workspace device buffer of at least gdn_prefill_workspace_bytes(T, N, Hq, Hv)
 *             bytes, 256-byte aligned (may be NULL when that size is 0); it holds
 *             the piece states of the segmented form (gdn_prefill_segmented),
 *             which the call takes when the (sequence, head) pairs would leave
 *             most SMs idle and the workspace is large enough
 * q, k, v, state and new_state need 16-byte alignment, cu_seqlens 8-byte.
 * A sequence of length 0 gets a zero final state (as in the definition).
 * cu_seqlens is read only on the device; values outside [0, T] are clamped.
 */
int gdn_prefill(const void *q, const void *k, const void *v, const float *state,
                const float *A_log, const void *a, const float *dt_bias, const void *b,
                const int64_t *cu_seqlens, float scale, void *output, float *new_state,
                int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                int64_t num_k_heads, int64_t num_v_heads, int64_t head_size, void *workspace,
                size_t workspace_bytes, void *stream);

/* Workspace bytes gdn_prefill wants for these sizes (0 when none). */
size_t gdn_prefill_workspace_bytes(int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                                   int64_t num_v_heads);

/*
 * Token-recurrent prefill on CUDA cores (no workspace).
 * Replaces gdn_prefill_recurrent_v1 (gdn_prefill/solution/python/cuda_recurrent_v1.cu:232-277).
 * Same arguments as gdn_prefill without the workspace.
 */
int gdn_prefill_recurrent(const void *q, const void *k, const void *v, const float *state,
                          const float *A_log, const void *a, const float *dt_bias, const void *b,
                          const int64_t *cu_seqlens, float scale, void *output, float *new_state,
                          int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                          int64_t num_k_heads, int64_t num_v_heads, int64_t head_size,
                          void *stream);

/* gdn_prefill_ex flags and paths */
#define GDN_PREFILL_QK_L2NORM 1   /* L2-normalise q and k per head: x / sqrt(sum x^2 + 1e-6) */
#define GDN_PREFILL_PATH_AUTO 0   /* the dispatch of gdn_prefill */
#define GDN_PREFILL_PATH_RECURRENT 1
#define GDN_PREFILL_PATH_CHUNKED 2

/*
 * gdn_prefill with options, without a workspace (so never the segmented form:
 * gdn_prefill_segmented takes one).  The
 * reference's prefill entry has no flags; GDN_PREFILL_QK_L2NORM is the in-kernel
 * q/k normalisation that FlashInfer's chunk_gated_delta_rule exposes as
 * use_qk_l2norm_in_kernel (rejected by the reference's baseline wrapper,
 * reference_solutions/.../flashinfer_wrapper_123ca6.md:271-273).  The chunked path
 * folds 1/|k_t| and 1/|q_t| into per-token factors instead of rescaling q and k.
 */
int gdn_prefill_ex(const void *q, const void *k, const void *v, const float *state,
                   const float *A_log, const void *a, const float *dt_bias, const void *b,
                   const int64_t *cu_seqlens, float scale, void *output, float *new_state,
                   int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                   int64_t num_k_heads, int64_t num_v_heads, int64_t head_size, int flags,
                   int path, void *stream);

/*
 * Head-sharded chunked prefill with the output all-gather fused into the kernel.
 * Replaces the pair "gdn_prefill_chunked on this rank's heads, then an NCCL
 * all_gather of o" (the multi-GPU form of gdn_prefill; the reference has no
 * multi-GPU path).  `output` is this rank's full [T, num_v_heads_out, 128] bf16
 * buffer; the call's num_v_heads heads (q/k/v/a/b/state/new_state hold only those)
 * are written at heads [head_offset, head_offset + num_v_heads) of it and of each
 * of the num_peers (<= 7) buffers in peer_outputs: device pointers, valid in this
 * process (peer-mapped, e.g. cudaIpcOpenMemHandle), of the other ranks' full output
 * buffers.  The kernel's own output stores go to every buffer; no collective runs.
 * The caller makes the writes visible (a barrier after every rank's call has
 * completed) before reading its buffer.  Buffers need 16-byte alignment.
 */
int gdn_prefill_chunked_peers(const void *q, const void *k, const void *v, const float *state,
                              const float *A_log, const void *a, const float *dt_bias,
                              const void *b, const int64_t *cu_seqlens, float scale,
                              void *output, float *new_state, int64_t total_seq_len,
                              int64_t num_seqs, int64_t num_q_heads, int64_t num_k_heads,
                              int64_t num_v_heads, int64_t head_size, int64_t num_v_heads_out,
                              int64_t head_offset, void *const *peer_outputs, int num_peers,
                              int segments, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Sequence-parallel (segmented) prefill; no counterpart in the reference, whose
 * chunked pipeline runs one state scan per (sequence, head).  Each sequence of
 * at least 2 * segments chunks is cut at chunk boundaries into `segments` pieces;
 * pass 1 runs piece 0 from the initial state and, for each middle piece g, its
 * final state from zero (F_g) and its transition matrix (P_g: the final state
 * from the identity with v = 0); S_{g+1} = S_g P_g + F_g gives the start states
 * (fp32); pass 2 runs pieces 1.. from them.  Four launches on the stream (three
 * for 2 pieces); the critical path is ~2/segments of the sequence.  Same arguments as
 * gdn_prefill plus flags (GDN_PREFILL_QK_L2NORM), segments (0 = automatic: each
 * sequence's count chosen on the device under gdn_prefill_segments' bound; 1 =
 * one chain per pair; 2..64 = that count for every sequence of at least 2 x that
 * many chunks) and a 256-byte aligned workspace of
 * gdn_prefill_segmented_workspace_bytes(N, Hv, segments) bytes (with segments 0,
 * sized for any bound: at most 1.5 x SMs x 64 KiB of piece states plus the
 * job tables).  gdn_prefill_chunked_peers takes the same three arguments.
 */
int gdn_prefill_segmented(const void *q, const void *k, const void *v, const float *state,
                          const float *A_log, const void *a, const float *dt_bias, const void *b,
                          const int64_t *cu_seqlens, float scale, void *output, float *new_state,
                          int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                          int64_t num_k_heads, int64_t num_v_heads, int64_t head_size, int flags,
                          int segments, void *workspace, size_t workspace_bytes, void *stream);
size_t gdn_prefill_segmented_workspace_bytes(int64_t num_seqs, int64_t num_v_heads, int segments);
/*
 * gdn_prefill_segmented without a workspace argument, for callers that cannot
 * allocate device memory per call: a host whose device memory belongs to its
 * own allocator (an inference server's arena, a plugin that is handed its
 * buffers and may not call cudaMalloc), or one that cannot afford the device
 * synchronisation cudaMalloc / cudaFree imply.  No counterpart in the reference
 * (its prefill entries take no workspace and allocate through torch).  The
 * scratch is a device array inside this library, GDN_NOALLOC_SCRATCH_BYTES
 * (16 MiB) on every GPU that loads it, kept until the process exits; a call
 * whose pieces need more (gdn_prefill_segmented_workspace_bytes) fails with
 * GDN_ERR_VALUE.  The first call on a device looks up the array's address on
 * that device (cudaGetSymbolAddress): make that first call before any stream
 * capture.  Every call shares the array, so calls that overlap on the GPU (on
 * two streams, or from two host threads) race; calls in one stream do not.
 * Nothing in it needs to start at zero (each call writes what it reads).  The
 * call allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
#define GDN_NOALLOC_SCRATCH_BYTES (16u << 20)
int gdn_prefill_segmented_noalloc(const void *q, const void *k, const void *v, const float *state,
                                  const float *A_log, const void *a, const float *dt_bias,
                                  const void *b, const int64_t *cu_seqlens, float scale,
                                  void *output, float *new_state, int64_t total_seq_len,
                                  int64_t num_seqs, int64_t num_q_heads, int64_t num_k_heads,
                                  int64_t num_v_heads, int64_t head_size, int flags, int segments,
                                  void *stream);

/* Upper bound of the automatic piece count for these sizes (1: the call is not
 * cut).  With segments 0 the call's first kernel picks, from the lengths on the
 * device, how many shares w (1 to 3) of a cut sequence its first piece takes and
 * each sequence's count under the bound: the shortest call time (pass 1, a fixed
 * cost of about six chunk-times for the extra launches, one chunk-time per
 * combine step, pass 2 = pass 1 / w; whole sequences within pass 1) whose pass-1
 * F/P jobs fit w waves of the SMs its piece-0 jobs leave free, whose pass 2 fits
 * one wave and whose piece states fit the workspace, with pieces of at least 2
 * chunks and counts of 1 or at least 3, and no cut at all unless it shortens the
 * call by a fifth.  The bound is 1 when the (sequence, head) pairs are more than
 * half the SMs or the call has fewer chunks in all than the shortest sequence
 * such a cut can take (23 chunks), else the largest G <= 16 with num_seqs *
 * num_v_heads * (G - 1) <= 2 x SMs and total_seq_len >= 4 G chunks. */
int gdn_prefill_segments(int64_t total_seq_len, int64_t num_seqs, int64_t num_v_heads);

/*
 * Chunk metadata (chunk size 64) for packed sequences.
 * Replaces prep_meta_v2 (gdn_prefill/solution/python/cuda_prep_meta_v2.cu:72-94),
 * without its N <= 256 limit.
 *   cu_seqlens     [N+1] int64 (device)
 *   chunk_offsets  [N+1] int32 (device, out): chunks before each sequence; [N] = total
 *   chunk_indices  [max_chunks, 2] int32 (device, out): (sequence, chunk) pairs
 */
int gdn_prep_meta(const int64_t *cu_seqlens, int64_t num_seqs, int32_t *chunk_offsets,
                  int32_t *chunk_indices, int64_t max_chunks, void *stream);

/*
 * Fused chunked (C = 64) prefill on tcgen05 tensor cores, whatever the size.
 * Replaces the reference's chunked pipeline (gdn_prefill/solution/python/chunk_v12.py:36-116:
 * prep_meta_v2, kkt_inv_uw_v1, h_v2b, o_v1) with one kernel that needs no workspace.
 * Same arguments as gdn_prefill_recurrent.
 */
int gdn_prefill_chunked(const void *q, const void *k, const void *v, const float *state,
                        const float *A_log, const void *a, const float *dt_bias, const void *b,
                        const int64_t *cu_seqlens, float scale, void *output, float *new_state,
                        int64_t total_seq_len, int64_t num_seqs, int64_t num_q_heads,
                        int64_t num_k_heads, int64_t num_v_heads, int64_t head_size, void *stream);

/*
 * Diagnostic form of gdn_prefill_chunked: also dumps the intermediates of one
 * chunk (dbg_seq, dbg_head, dbg_chunk) into `debug` (fp32, at least
 * gdn_prefill_chunked_debug_floats() elements): gamma[64], beta[64], A[64x64],
 * P[64x64], T[64x64], U[64x128], W[64x128], Vn[64x128], QS[64x128], PV[64x128],
 * state after the chunk [128x128].  The in-kernel counterpart of the reference's
 * optional %globaltimer profiler argument (cuda_h_v2b.cu:56-121,829-896).
 */
int gdn_prefill_chunked_debug(const void *q, const void *k, const void *v, const float *state,
                              const float *A_log, const void *a, const float *dt_bias,
                              const void *b, const int64_t *cu_seqlens, float scale, void *output,
                              float *new_state, int64_t total_seq_len, int64_t num_seqs,
                              int64_t num_q_heads, int64_t num_k_heads, int64_t num_v_heads,
                              int64_t head_size, float *debug, int64_t debug_floats,
                              int64_t dbg_seq, int64_t dbg_head, int64_t dbg_chunk, void *stream);
int64_t gdn_prefill_chunked_debug_floats(void);

/*
 * Device status word.  A kernel that gives up on a bounded wait (an mbarrier
 * that does not complete within 2 s) sets a bit here and returns instead of
 * hanging: bit 0 = chunked prefill, bit 1 = gdn_wait_probe.  Reads the word of
 * the current device (synchronising), optionally clearing it.  No reference
 * counterpart: the reference relies on cudaGetLastError only
 * (gdn_decode_small_batch.cu:223-227).
 */
int gdn_read_status(uint32_t *status, int clear);

/* Launches one CTA that waits on an mbarrier nothing arrives on, for at most
 * timeout_ns (<= 5 s); *result (device memory, may be NULL) becomes 0 on
 * timeout.  Exercises the timeout path without faulting or hanging the GPU. */
int gdn_wait_probe(uint64_t timeout_ns, uint32_t *result, void *stream);

/* Upper bound on the number of 64-token chunks of T tokens in N sequences
 * (N + (T - N) / 64 for T >= N; the reference's bound in chunk_v12.py:53). */
int64_t gdn_chunk_upper_bound(int64_t total_seq_len, int64_t num_seqs);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
