// TVM-FFI module of the gdn_b200 kernels: the native binding the reference's
// Solutions load with tvm_ffi.load_module (gdn_decode/solution/python/
// gdn_decode_kernel_cuda_small_batch.py, gdn_prefill/solution/python/chunk_v12.py:17-33,
// cuda_recurrent_v1.py), exported with TVM_FFI_DLL_EXPORT_TYPED_FUNC over DLPack
// TensorViews in the style of the reference's other/tvm_ffi_example.  Every export
// validates its tensors (device, contiguity, rank, dtype, shape) with the
// reference's exception kinds (ValueError for device/layout/shape, TypeError for
// dtypes; gdn_decode/solution/python/gdn_decode_utils.h:16-122), then makes one
// call of the C ABI (include/gdn_b200.h) on the environment stream of the
// tensors' device (TVMFFIEnvGetStream: the torch current stream when called from
// torch) under a device guard.  C-ABI failures become ValueError / TypeError /
// RuntimeError with the library's message.  Nothing is allocated here: the
// caller passes every output, as the reference's FFI functions expect.
//
// Exports:
//   gdn_decode_small_batch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
//       name and arguments of gdn_decode_small_batch.cu:194-232 (state required)
//   gdn_decode(q, k, v, state?, A_log, a, dt_bias, b, scale, output, new_state)
//       the same with an optional state (None = zero initial state)
//   gdn_prefill_recurrent_v1(q, k, v, state?, A_log, a, dt_bias, b, cu_seqlens, scale,
//                            output, new_state)
//       name and arguments of cuda_recurrent_v1.cu:232-281
//   gdn_prefill(q, k, v, state?, A_log, a, dt_bias, b, cu_seqlens, scale, output,
//               new_state, workspace?)
//       the dispatch of gdn_prefill_mix.py:13-38 (recurrent / chunked / segmented);
//       workspace: uint8 device tensor of gdn_prefill_workspace_bytes (optional)
//   gdn_prefill_chunked(q, k, v, state?, A_log, a, dt_bias, b, cu_seqlens, scale,
//                       output, new_state)
//       the fused chunked kernel (the chunk_v12.py:36-116 pipeline in one launch)
//   prep_meta_v2(cu_seqlens, chunk_indices, chunk_offsets)
//       name and argument order of cuda_prep_meta_v2.cu:72-96 (no N <= 256 limit)
//   gdn_prefill_workspace_bytes(total_seq_len, num_seqs, num_q_heads, num_v_heads) -> int
#include <cuda_runtime.h>

#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/extra/cuda/device_guard.h>
#include <tvm/ffi/tvm_ffi.h>

#include "gdn_b200.h"

namespace {

namespace ffi = tvm::ffi;
using ffi::Optional;
using ffi::TensorView;

constexpr int64_t kHead = 128;
constexpr DLDataType kBf16{kDLBfloat, 16, 1};
constexpr DLDataType kF32{kDLFloat, 32, 1};
constexpr DLDataType kI64{kDLInt, 64, 1};
constexpr DLDataType kI32{kDLInt, 32, 1};
constexpr DLDataType kU8{kDLUInt, 8, 1};

bool same_type(DLDataType a, DLDataType b) {
  return a.code == b.code && a.bits == b.bits && a.lanes == b.lanes;
}

const char* type_name(DLDataType t) {
  if (same_type(t, kBf16)) return "bfloat16";
  if (same_type(t, kF32)) return "float32";
  if (same_type(t, kI64)) return "int64";
  if (same_type(t, kI32)) return "int32";
  if (same_type(t, kU8)) return "uint8";
  return "another dtype";
}

// The data pointer of a DLPack tensor includes its byte offset.
void* ptr(const TensorView& t) {
  return static_cast<char*>(t.data_ptr()) + t.byte_offset();
}

void cuda_contig(const TensorView& t, const char* name) {
  TVM_FFI_CHECK(t.device().device_type == kDLCUDA, ValueError) << name << " must be a CUDA tensor";
  TVM_FFI_CHECK(t.IsContiguous(), ValueError) << name << " must be contiguous";
}

void rank(const TensorView& t, const char* name, int d) {
  TVM_FFI_CHECK(t.ndim() == d, ValueError) << name << " must be a " << d << "D tensor";
}

void dtype(const TensorView& t, const char* name, DLDataType want) {
  TVM_FFI_CHECK(same_type(t.dtype(), want), TypeError)
      << name << " must be " << type_name(want) << " (got " << type_name(t.dtype()) << ")";
}

void same_device(const TensorView& ref, const TensorView& t, const char* name) {
  TVM_FFI_CHECK(t.device().device_type == ref.device().device_type &&
                    t.device().device_id == ref.device().device_id,
                ValueError)
      << "q and " << name << " must be on the same device";
}

void shape(const TensorView& t, const char* name, std::initializer_list<int64_t> dims,
           const char* text) {
  bool ok = t.ndim() == static_cast<int>(dims.size());
  int i = 0;
  for (int64_t d : dims) ok = ok && t.size(i++) == d;
  TVM_FFI_CHECK(ok, ValueError) << name << " must have shape " << text;
}

void tensor(const TensorView& t, const TensorView& q, const char* name, int nd, DLDataType dt) {
  cuda_contig(t, name);
  rank(t, name, nd);
  dtype(t, name, dt);
  same_device(q, t, name);
}

void check_rc(int rc, const char* what) {
  if (rc == GDN_OK) return;
  const char* msg = gdn_last_error();
  TVM_FFI_CHECK(rc != GDN_ERR_VALUE, ValueError) << what << ": " << msg;
  TVM_FFI_CHECK(rc != GDN_ERR_TYPE, TypeError) << what << ": " << msg;
  TVM_FFI_THROW(RuntimeError) << what << ": " << msg;
}

void* env_stream(const TensorView& t) {
  return TVMFFIEnvGetStream(t.device().device_type, t.device().device_id);
}

// ---------------------------------------------------------------- decode
void decode_impl(const TensorView& q, const TensorView& k, const TensorView& v,
                 const TensorView* state, const TensorView& A_log, const TensorView& a,
                 const TensorView& dt_bias, const TensorView& b, double scale,
                 const TensorView& output, const TensorView& new_state) {
  tensor(q, q, "q", 4, kBf16);
  tensor(k, q, "k", 4, kBf16);
  tensor(v, q, "v", 4, kBf16);
  tensor(A_log, q, "A_log", 1, kF32);
  tensor(a, q, "a", 3, kBf16);
  tensor(dt_bias, q, "dt_bias", 1, kF32);
  tensor(b, q, "b", 3, kBf16);
  const int64_t B = q.size(0), T = q.size(1), Hq = q.size(2), Hk = k.size(2), Hv = v.size(2);
  TVM_FFI_CHECK(k.size(0) == B && v.size(0) == B, ValueError) << "batch mismatch among q/k/v";
  TVM_FFI_CHECK(k.size(1) == T && v.size(1) == T, ValueError)
      << "sequence length mismatch among q/k/v";
  TVM_FFI_CHECK(T == 1, ValueError) << "decode requires T=1";
  TVM_FFI_CHECK(q.size(3) == kHead && k.size(3) == kHead && v.size(3) == kHead, ValueError)
      << "head size must be 128";
  TVM_FFI_CHECK(Hk == Hq, ValueError) << "num_k_heads must equal num_q_heads";
  TVM_FFI_CHECK(Hq > 0 && Hv % Hq == 0, ValueError) << "HV must be divisible by Hq";
  shape(a, "a", {B, T, Hv}, "[B, T, HV]");
  shape(b, "b", {B, T, Hv}, "[B, T, HV]");
  shape(A_log, "A_log", {Hv}, "[HV]");
  shape(dt_bias, "dt_bias", {Hv}, "[HV]");
  if (state) {
    tensor(*state, q, "state", 4, kF32);
    shape(*state, "state", {B, Hv, kHead, kHead}, "[B, HV, V, K]");
  }
  tensor(output, q, "output", 4, kBf16);
  shape(output, "output", {B, T, Hv, kHead}, "[B, T, HV, V]");
  tensor(new_state, q, "new_state", 4, kF32);
  shape(new_state, "new_state", {B, Hv, kHead, kHead}, "[B, HV, V, K]");
  ffi::CUDADeviceGuard guard(q.device().device_id);
  check_rc(gdn_decode(ptr(q), ptr(k), ptr(v), state ? static_cast<const float*>(ptr(*state)) : nullptr,
                      static_cast<const float*>(ptr(A_log)), ptr(a),
                      static_cast<const float*>(ptr(dt_bias)), ptr(b), static_cast<float>(scale),
                      ptr(output), static_cast<float*>(ptr(new_state)), B, Hq, Hk, Hv, kHead,
                      env_stream(q)),
           "gdn_decode");
}

void DecodeSmallBatch(TensorView q, TensorView k, TensorView v, TensorView state, TensorView A_log,
                      TensorView a, TensorView dt_bias, TensorView b, double scale,
                      TensorView output, TensorView new_state) {
  decode_impl(q, k, v, &state, A_log, a, dt_bias, b, scale, output, new_state);
}

void Decode(TensorView q, TensorView k, TensorView v, Optional<TensorView> state,
            TensorView A_log, TensorView a, TensorView dt_bias, TensorView b, double scale,
            TensorView output, TensorView new_state) {
  if (state.has_value()) {
    const TensorView s = state.value();
    decode_impl(q, k, v, &s, A_log, a, dt_bias, b, scale, output, new_state);
  } else {
    decode_impl(q, k, v, nullptr, A_log, a, dt_bias, b, scale, output, new_state);
  }
}

// ---------------------------------------------------------------- prefill
enum class PrefillPath { kAuto, kRecurrent, kChunked };

void prefill_impl(PrefillPath path, const TensorView& q, const TensorView& k, const TensorView& v,
                  const Optional<TensorView>& state, const TensorView& A_log, const TensorView& a,
                  const TensorView& dt_bias, const TensorView& b, const TensorView& cu_seqlens,
                  double scale, const TensorView& output, const TensorView& new_state,
                  const Optional<TensorView>& workspace) {
  tensor(q, q, "q", 3, kBf16);
  tensor(k, q, "k", 3, kBf16);
  tensor(v, q, "v", 3, kBf16);
  tensor(A_log, q, "A_log", 1, kF32);
  tensor(a, q, "a", 2, kBf16);
  tensor(dt_bias, q, "dt_bias", 1, kF32);
  tensor(b, q, "b", 2, kBf16);
  // cu_seqlens is int64 in the definition; the kernels read it on the device
  tensor(cu_seqlens, q, "cu_seqlens", 1, kI64);
  const int64_t T = q.size(0), Hq = q.size(1), Hk = k.size(1), Hv = v.size(1);
  const int64_t N = cu_seqlens.size(0) - 1;
  TVM_FFI_CHECK(N >= 0, ValueError) << "cu_seqlens must have at least one element";
  TVM_FFI_CHECK(k.size(0) == T && v.size(0) == T, ValueError) << "token count mismatch among q/k/v";
  TVM_FFI_CHECK(q.size(2) == kHead && k.size(2) == kHead && v.size(2) == kHead, ValueError)
      << "head size must be 128";
  TVM_FFI_CHECK(Hk == Hq, ValueError) << "num_k_heads must equal num_q_heads";
  TVM_FFI_CHECK(Hq > 0 && Hv % Hq == 0, ValueError) << "HV must be divisible by Hq";
  shape(a, "a", {T, Hv}, "[T, HV]");
  shape(b, "b", {T, Hv}, "[T, HV]");
  shape(A_log, "A_log", {Hv}, "[HV]");
  shape(dt_bias, "dt_bias", {Hv}, "[HV]");
  const float* sp = nullptr;
  if (state.has_value()) {
    const TensorView s = state.value();
    tensor(s, q, "state", 4, kF32);
    shape(s, "state", {N, Hv, kHead, kHead}, "[N, HV, V, K]");
    sp = static_cast<const float*>(ptr(s));
  }
  tensor(output, q, "output", 3, kBf16);
  shape(output, "output", {T, Hv, kHead}, "[T, HV, V]");
  tensor(new_state, q, "new_state", 4, kF32);
  shape(new_state, "new_state", {N, Hv, kHead, kHead}, "[N, HV, V, K]");
  void* ws = nullptr;
  size_t ws_bytes = 0;
  if (workspace.has_value()) {
    const TensorView w = workspace.value();
    tensor(w, q, "workspace", 1, kU8);
    ws = ptr(w);
    ws_bytes = static_cast<size_t>(w.size(0));
  }
  ffi::CUDADeviceGuard guard(q.device().device_id);
  void* stream = env_stream(q);
  const float sc = static_cast<float>(scale);
  const float* al = static_cast<const float*>(ptr(A_log));
  const float* dt = static_cast<const float*>(ptr(dt_bias));
  const int64_t* cu = static_cast<const int64_t*>(ptr(cu_seqlens));
  float* ns = static_cast<float*>(ptr(new_state));
  switch (path) {
    case PrefillPath::kRecurrent:
      check_rc(gdn_prefill_recurrent(ptr(q), ptr(k), ptr(v), sp, al, ptr(a), dt, ptr(b), cu, sc,
                                     ptr(output), ns, T, N, Hq, Hk, Hv, kHead, stream),
               "gdn_prefill_recurrent");
      break;
    case PrefillPath::kChunked:
      check_rc(gdn_prefill_chunked(ptr(q), ptr(k), ptr(v), sp, al, ptr(a), dt, ptr(b), cu, sc,
                                   ptr(output), ns, T, N, Hq, Hk, Hv, kHead, stream),
               "gdn_prefill_chunked");
      break;
    default:
      check_rc(gdn_prefill(ptr(q), ptr(k), ptr(v), sp, al, ptr(a), dt, ptr(b), cu, sc, ptr(output),
                           ns, T, N, Hq, Hk, Hv, kHead, ws, ws_bytes, stream),
               "gdn_prefill");
  }
}

void PrefillRecurrentV1(TensorView q, TensorView k, TensorView v, Optional<TensorView> state,
                        TensorView A_log, TensorView a, TensorView dt_bias, TensorView b,
                        TensorView cu_seqlens, double scale, TensorView output,
                        TensorView new_state) {
  prefill_impl(PrefillPath::kRecurrent, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
               output, new_state, Optional<TensorView>());
}

void Prefill(TensorView q, TensorView k, TensorView v, Optional<TensorView> state,
             TensorView A_log, TensorView a, TensorView dt_bias, TensorView b,
             TensorView cu_seqlens, double scale, TensorView output, TensorView new_state,
             Optional<TensorView> workspace) {
  prefill_impl(PrefillPath::kAuto, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
               output, new_state, workspace);
}

void PrefillChunked(TensorView q, TensorView k, TensorView v, Optional<TensorView> state,
                    TensorView A_log, TensorView a, TensorView dt_bias, TensorView b,
                    TensorView cu_seqlens, double scale, TensorView output,
                    TensorView new_state) {
  prefill_impl(PrefillPath::kChunked, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
               output, new_state, Optional<TensorView>());
}

// chunk metadata, argument order of the reference's prep_meta_v2
void PrepMetaV2(TensorView cu_seqlens, TensorView chunk_indices, TensorView chunk_offsets) {
  tensor(cu_seqlens, cu_seqlens, "cu_seqlens", 1, kI64);
  tensor(chunk_indices, cu_seqlens, "chunk_indices", 2, kI32);
  tensor(chunk_offsets, cu_seqlens, "chunk_offsets", 1, kI32);
  const int64_t N = cu_seqlens.size(0) - 1;
  TVM_FFI_CHECK(N >= 0, ValueError) << "cu_seqlens must have at least one element";
  TVM_FFI_CHECK(chunk_offsets.size(0) == N + 1, ValueError) << "chunk_offsets must have shape [N+1]";
  TVM_FFI_CHECK(chunk_indices.size(1) == 2, ValueError) << "chunk_indices must have shape [C, 2]";
  ffi::CUDADeviceGuard guard(cu_seqlens.device().device_id);
  check_rc(gdn_prep_meta(static_cast<const int64_t*>(ptr(cu_seqlens)), N,
                         static_cast<int32_t*>(ptr(chunk_offsets)),
                         static_cast<int32_t*>(ptr(chunk_indices)), chunk_indices.size(0),
                         env_stream(cu_seqlens)),
           "gdn_prep_meta");
}

int64_t PrefillWorkspaceBytes(int64_t T, int64_t N, int64_t Hq, int64_t Hv) {
  return static_cast<int64_t>(gdn_prefill_workspace_bytes(T, N, Hq, Hv));
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_decode_small_batch, DecodeSmallBatch);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_decode, Decode);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_prefill_recurrent_v1, PrefillRecurrentV1);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_prefill, Prefill);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_prefill_chunked, PrefillChunked);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(prep_meta_v2, PrepMetaV2);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_prefill_workspace_bytes, PrefillWorkspaceBytes);
