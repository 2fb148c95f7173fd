// Native Python binding of the C ABI (include/gdn_b200.h) for torch tensors: the
// role TVM-FFI plays for the reference (gdn_decode/solution/python/gdn_decode_utils.h,
// gdn_prefill/solution/python/cuda_utils.h).  Each entry point checks the tensors'
// device, layout, rank and dtype, allocates the outputs the caller did not pass
// from the torch caching allocator, and makes one C-ABI call on the tensors'
// current CUDA stream.  Checks raise the same exception types as the Python
// checks in gdn_b200/_checks.py (ValueError for device/layout/shape, TypeError for
// dtypes); C-ABI error codes map GDN_ERR_VALUE -> ValueError, GDN_ERR_TYPE ->
// TypeError, GDN_ERR_CUDA -> RuntimeError.  Doing this in C++ takes the host cost
// of a call from ~30 us (Python checks + ctypes) to a few microseconds, which is
// most of the latency of a small decode or prefill call.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "gdn_b200.h"

namespace {

constexpr int64_t kHead = 128;

void cuda_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK_VALUE(t.is_contiguous(), name, " must be contiguous");
}

void rank(const at::Tensor& t, const char* name, int64_t d) {
  TORCH_CHECK_VALUE(t.dim() == d, name, " must be a ", d, "D tensor");
}

void dtype(const at::Tensor& t, const char* name, at::ScalarType s) {
  TORCH_CHECK_TYPE(t.scalar_type() == s, name, " must be ",
                   s == at::kBFloat16 ? "bfloat16" : s == at::kFloat ? "float32" : "int64");
}

void same_device(const at::Tensor& ref, const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.device() == ref.device(), "q and ", name, " must be on the same device");
}

void check_rc(int rc, const char* what) {
  if (rc == GDN_OK) return;
  const char* msg = gdn_last_error();
  TORCH_CHECK_VALUE(rc != GDN_ERR_VALUE, what, ": ", msg);
  TORCH_CHECK_TYPE(rc != GDN_ERR_TYPE, what, ": ", msg);
  TORCH_CHECK(false, what, ": ", msg);
}

const float* state_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr<float>() : nullptr;
}

// decode: q, k [B,1,Hq,128] bf16; v [B,1,Hv,128] bf16; state [B,Hv,128,128] fp32 or
// None; A_log, dt_bias [Hv] fp32; a, b [B,1,Hv] bf16 -> (output, new_state).
// output / new_state: destinations (new_state may be state itself: in place).
std::tuple<at::Tensor, at::Tensor> decode(const at::Tensor& q, const at::Tensor& k,
                                          const at::Tensor& v,
                                          const c10::optional<at::Tensor>& state,
                                          const at::Tensor& A_log, const at::Tensor& a,
                                          const at::Tensor& dt_bias, const at::Tensor& b,
                                          double scale, c10::optional<at::Tensor> output,
                                          c10::optional<at::Tensor> new_state) {
  const std::pair<const at::Tensor*, const char*> ins[] = {
      {&q, "q"}, {&k, "k"}, {&v, "v"}, {&A_log, "A_log"}, {&a, "a"}, {&dt_bias, "dt_bias"}, {&b, "b"}};
  for (const auto& [t, n] : ins) cuda_contig(*t, n);
  rank(q, "q", 4);
  rank(k, "k", 4);
  rank(v, "v", 4);
  rank(A_log, "A_log", 1);
  rank(a, "a", 3);
  rank(dt_bias, "dt_bias", 1);
  rank(b, "b", 3);
  for (const auto& [t, n] : ins) same_device(q, *t, n);
  dtype(q, "q", at::kBFloat16);
  dtype(k, "k", at::kBFloat16);
  dtype(v, "v", at::kBFloat16);
  dtype(a, "a", at::kBFloat16);
  dtype(b, "b", at::kBFloat16);
  dtype(A_log, "A_log", at::kFloat);
  dtype(dt_bias, "dt_bias", at::kFloat);
  const int64_t B = q.size(0), T = q.size(1), Hq = q.size(2), Hk = k.size(2), Hv = v.size(2);
  TORCH_CHECK_VALUE(k.size(0) == B && v.size(0) == B, "batch mismatch among q/k/v");
  TORCH_CHECK_VALUE(k.size(1) == T && v.size(1) == T, "sequence length mismatch among q/k/v");
  TORCH_CHECK_VALUE(T == 1, "decode requires T=1");
  TORCH_CHECK_VALUE(q.size(3) == kHead && k.size(3) == kHead && v.size(3) == kHead,
                    "head size must be 128");
  TORCH_CHECK_VALUE(Hk == Hq, "num_k_heads must equal num_q_heads");
  TORCH_CHECK_VALUE(Hq > 0 && Hv % Hq == 0, "HV must be divisible by Hq");
  TORCH_CHECK_VALUE(a.sizes() == at::IntArrayRef({B, T, Hv}), "a must have shape [B, T, HV]");
  TORCH_CHECK_VALUE(b.sizes() == at::IntArrayRef({B, T, Hv}), "b must have shape [B, T, HV]");
  TORCH_CHECK_VALUE(A_log.size(0) == Hv, "A_log must have shape [HV]");
  TORCH_CHECK_VALUE(dt_bias.size(0) == Hv, "dt_bias must have shape [HV]");
  if (state.has_value()) {
    cuda_contig(*state, "state");
    rank(*state, "state", 4);
    dtype(*state, "state", at::kFloat);
    same_device(q, *state, "state");
    TORCH_CHECK_VALUE(state->sizes() == at::IntArrayRef({B, Hv, kHead, kHead}),
                      "state must have shape [B, HV, V, K]");
  }
  if (output.has_value()) {
    cuda_contig(*output, "output");
    rank(*output, "output", 4);
    dtype(*output, "output", at::kBFloat16);
    same_device(q, *output, "output");
    TORCH_CHECK_VALUE(output->sizes() == at::IntArrayRef({B, T, Hv, kHead}),
                      "output must have shape [B, T, HV, V]");
  } else {
    output = at::empty_like(v);
  }
  if (new_state.has_value()) {
    cuda_contig(*new_state, "new_state");
    rank(*new_state, "new_state", 4);
    dtype(*new_state, "new_state", at::kFloat);
    same_device(q, *new_state, "new_state");
    TORCH_CHECK_VALUE(new_state->sizes() == at::IntArrayRef({B, Hv, kHead, kHead}),
                      "new_state must have shape [B, HV, V, K]");
  } else {
    new_state = at::empty({B, Hv, kHead, kHead}, v.options().dtype(at::kFloat));
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  check_rc(gdn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), state_ptr(state), A_log.data_ptr<float>(),
                      a.data_ptr(), dt_bias.data_ptr<float>(), b.data_ptr(), static_cast<float>(scale),
                      output->data_ptr(), new_state->data_ptr<float>(), B, Hq, Hk, Hv, kHead, stream),
           "gdn_decode");
  return {*output, *new_state};
}

// prefill: q, k [T,Hq,128] bf16; v [T,Hv,128] bf16; state [N,Hv,128,128] fp32 or
// None; a, b [T,Hv] bf16; cu_seqlens [N+1] int64 -> (output, new_state).
// path: 0 = the default dispatch (gdn_prefill: recurrent, segmented or chunked),
// 1 = token-recurrent kernel, 2 = chunked kernel, 3 = segmented with `segments`
// pieces (0 = automatic); qk_l2norm: in-kernel q/k L2 normalisation.  The
// segmented form's workspace comes from the caching allocator.
std::tuple<at::Tensor, at::Tensor> prefill(const at::Tensor& q, const at::Tensor& k,
                                           const at::Tensor& v,
                                           const c10::optional<at::Tensor>& state,
                                           const at::Tensor& A_log, const at::Tensor& a,
                                           const at::Tensor& dt_bias, const at::Tensor& b,
                                           const at::Tensor& cu_seqlens, double scale,
                                           c10::optional<at::Tensor> output,
                                           c10::optional<at::Tensor> new_state, int64_t path,
                                           bool qk_l2norm, int64_t segments) {
  const std::pair<const at::Tensor*, const char*> ins[] = {
      {&q, "q"}, {&k, "k"},           {&v, "v"}, {&A_log, "A_log"}, {&a, "a"}, {&dt_bias, "dt_bias"},
      {&b, "b"}, {&cu_seqlens, "cu_seqlens"}};
  for (const auto& [t, n] : ins) cuda_contig(*t, n);
  rank(q, "q", 3);
  rank(k, "k", 3);
  rank(v, "v", 3);
  rank(A_log, "A_log", 1);
  rank(a, "a", 2);
  rank(dt_bias, "dt_bias", 1);
  rank(b, "b", 2);
  rank(cu_seqlens, "cu_seqlens", 1);
  const int64_t T = q.size(0), Hq = q.size(1), Nseq = cu_seqlens.size(0) - 1;
  const int64_t Hk = k.size(1), Hv = v.size(1);
  TORCH_CHECK_VALUE(Nseq > 0, "must have at least one sequence");
  TORCH_CHECK_VALUE(path >= 0 && path <= 3,
                    "path must be 0 (auto), 1 (recurrent), 2 (chunked) or 3 (segmented)");
  TORCH_CHECK_VALUE(segments >= 0 && segments <= 64, "segments must be in [0, 64]");
  TORCH_CHECK_VALUE(q.size(2) == kHead && k.size(2) == kHead && v.size(2) == kHead,
                    "head size must be 128");
  TORCH_CHECK_VALUE(k.size(0) == T && v.size(0) == T, "k/v shape mismatch");
  TORCH_CHECK_VALUE(Hk == Hq, "num_k_heads must equal num_q_heads");
  TORCH_CHECK_VALUE(Hq > 0 && Hv % Hq == 0, "num_v_heads must be divisible by num_q_heads");
  TORCH_CHECK_VALUE(a.sizes() == at::IntArrayRef({T, Hv}), "a shape mismatch");
  TORCH_CHECK_VALUE(b.sizes() == at::IntArrayRef({T, Hv}), "b shape mismatch");
  TORCH_CHECK_VALUE(A_log.size(0) == Hv && dt_bias.size(0) == Hv,
                    "A_log / dt_bias must have shape [HV]");
  dtype(q, "q", at::kBFloat16);
  dtype(k, "k", at::kBFloat16);
  dtype(v, "v", at::kBFloat16);
  dtype(a, "a", at::kBFloat16);
  dtype(b, "b", at::kBFloat16);
  dtype(A_log, "A_log", at::kFloat);
  dtype(dt_bias, "dt_bias", at::kFloat);
  dtype(cu_seqlens, "cu_seqlens", at::kLong);
  for (const auto& [t, n] : ins) same_device(q, *t, n);
  if (state.has_value()) {
    cuda_contig(*state, "state");
    rank(*state, "state", 4);
    dtype(*state, "state", at::kFloat);
    same_device(q, *state, "state");
    TORCH_CHECK_VALUE(state->sizes() == at::IntArrayRef({Nseq, Hv, kHead, kHead}),
                      "state shape mismatch");
  }
  if (output.has_value()) {
    cuda_contig(*output, "output");
    rank(*output, "output", 3);
    dtype(*output, "output", at::kBFloat16);
    same_device(q, *output, "output");
    TORCH_CHECK_VALUE(output->sizes() == at::IntArrayRef({T, Hv, kHead}), "output shape mismatch");
  } else {
    output = at::empty_like(v);
  }
  if (new_state.has_value()) {
    cuda_contig(*new_state, "new_state");
    rank(*new_state, "new_state", 4);
    dtype(*new_state, "new_state", at::kFloat);
    same_device(q, *new_state, "new_state");
    TORCH_CHECK_VALUE(new_state->sizes() == at::IntArrayRef({Nseq, Hv, kHead, kHead}),
                      "new_state shape mismatch");
  } else {
    new_state = at::empty({Nseq, Hv, kHead, kHead}, v.options().dtype(at::kFloat));
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  // the segmented form: automatic (segments 0: the device picks each sequence's
  // pieces under gdn_prefill_segments' bound) or a forced count
  const bool cut = (path == 0 && gdn_prefill_segments(T, Nseq, Hv) > 1) || path == 3;
  const int flags = qk_l2norm ? GDN_PREFILL_QK_L2NORM : 0;
  if (cut) {
    const int G = path == 3 ? static_cast<int>(segments) : 0;
    const size_t ws_bytes = G > 0 ? gdn_prefill_segmented_workspace_bytes(Nseq, Hv, G)
                                  : gdn_prefill_workspace_bytes(T, Nseq, Hq, Hv);
    at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(at::kByte));
    check_rc(gdn_prefill_segmented(q.data_ptr(), k.data_ptr(), v.data_ptr(), state_ptr(state),
                                   A_log.data_ptr<float>(), a.data_ptr(), dt_bias.data_ptr<float>(),
                                   b.data_ptr(), cu_seqlens.data_ptr<int64_t>(),
                                   static_cast<float>(scale), output->data_ptr(),
                                   new_state->data_ptr<float>(), T, Nseq, Hq, Hk, Hv, kHead, flags,
                                   G, ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream),
             "gdn_prefill_segmented");
    return {*output, *new_state};
  }
  check_rc(gdn_prefill_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), state_ptr(state),
                          A_log.data_ptr<float>(), a.data_ptr(), dt_bias.data_ptr<float>(),
                          b.data_ptr(), cu_seqlens.data_ptr<int64_t>(), static_cast<float>(scale),
                          output->data_ptr(), new_state->data_ptr<float>(), T, Nseq, Hq, Hk, Hv,
                          kHead, flags, path == 3 ? GDN_PREFILL_PATH_CHUNKED : static_cast<int>(path),
                          stream),
           "gdn_prefill_ex");
  return {*output, *new_state};
}

// pooled multi-token decode: q, k [B,T,Hq,128] bf16; v [B,T,Hv,128] bf16; a, b
// [B,T,Hv] bf16; state_pool [P,Hv,128,128] fp32 or bf16 (updated in place);
// in_slots / out_slots [B] int32; intermediate: None or [B,T,Hv,128,128] in the
// pool's dtype -> output [B,T,Hv,128] bf16.
at::Tensor decode_pool(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                       const at::Tensor& A_log, const at::Tensor& a, const at::Tensor& dt_bias,
                       const at::Tensor& b, double scale, const at::Tensor& state_pool,
                       const at::Tensor& in_slots, const c10::optional<at::Tensor>& out_slots,
                       const c10::optional<at::Tensor>& intermediate, bool qk_l2norm,
                       bool no_state_update, c10::optional<at::Tensor> output) {
  const std::pair<const at::Tensor*, const char*> ins[] = {
      {&q, "q"}, {&k, "k"}, {&v, "v"}, {&A_log, "A_log"}, {&a, "a"}, {&dt_bias, "dt_bias"},
      {&b, "b"}, {&state_pool, "state_pool"}, {&in_slots, "in_slots"}};
  for (const auto& [t, n] : ins) cuda_contig(*t, n);
  rank(q, "q", 4);
  rank(k, "k", 4);
  rank(v, "v", 4);
  rank(A_log, "A_log", 1);
  rank(a, "a", 3);
  rank(dt_bias, "dt_bias", 1);
  rank(b, "b", 3);
  rank(state_pool, "state_pool", 4);
  rank(in_slots, "in_slots", 1);
  for (const auto& [t, n] : ins) same_device(q, *t, n);
  dtype(q, "q", at::kBFloat16);
  dtype(k, "k", at::kBFloat16);
  dtype(v, "v", at::kBFloat16);
  dtype(a, "a", at::kBFloat16);
  dtype(b, "b", at::kBFloat16);
  dtype(A_log, "A_log", at::kFloat);
  dtype(dt_bias, "dt_bias", at::kFloat);
  TORCH_CHECK_TYPE(state_pool.scalar_type() == at::kFloat || state_pool.scalar_type() == at::kBFloat16,
                   "state_pool must be float32 or bfloat16");
  TORCH_CHECK_TYPE(in_slots.scalar_type() == at::kInt, "in_slots must be int32");
  const int64_t B = q.size(0), T = q.size(1), Hq = q.size(2), Hk = k.size(2), Hv = v.size(2);
  const int64_t P = state_pool.size(0);
  TORCH_CHECK_VALUE(k.size(0) == B && v.size(0) == B, "batch mismatch among q/k/v");
  TORCH_CHECK_VALUE(k.size(1) == T && v.size(1) == T, "sequence length mismatch among q/k/v");
  TORCH_CHECK_VALUE(T >= 1, "need at least one token per sequence");
  TORCH_CHECK_VALUE(q.size(3) == kHead && k.size(3) == kHead && v.size(3) == kHead,
                    "head size must be 128");
  TORCH_CHECK_VALUE(Hk == Hq, "num_k_heads must equal num_q_heads");
  TORCH_CHECK_VALUE(Hq > 0 && Hv % Hq == 0, "HV must be divisible by Hq");
  TORCH_CHECK_VALUE(a.sizes() == at::IntArrayRef({B, T, Hv}), "a must have shape [B, T, HV]");
  TORCH_CHECK_VALUE(b.sizes() == at::IntArrayRef({B, T, Hv}), "b must have shape [B, T, HV]");
  TORCH_CHECK_VALUE(A_log.size(0) == Hv && dt_bias.size(0) == Hv,
                    "A_log / dt_bias must have shape [HV]");
  TORCH_CHECK_VALUE(state_pool.sizes() == at::IntArrayRef({P, Hv, kHead, kHead}),
                    "state_pool must have shape [pool_size, HV, V, K]");
  TORCH_CHECK_VALUE(in_slots.size(0) == B, "in_slots must have shape [B]");
  if (out_slots.has_value()) {
    cuda_contig(*out_slots, "out_slots");
    rank(*out_slots, "out_slots", 1);
    same_device(q, *out_slots, "out_slots");
    TORCH_CHECK_TYPE(out_slots->scalar_type() == at::kInt, "out_slots must be int32");
    TORCH_CHECK_VALUE(out_slots->size(0) == B, "out_slots must have shape [B]");
  }
  if (intermediate.has_value()) {
    cuda_contig(*intermediate, "intermediate");
    same_device(q, *intermediate, "intermediate");
    TORCH_CHECK_TYPE(intermediate->scalar_type() == state_pool.scalar_type(),
                     "intermediate must have the state_pool dtype");
    TORCH_CHECK_VALUE(intermediate->sizes() == at::IntArrayRef({B, T, Hv, kHead, kHead}),
                      "intermediate must have shape [B, T, HV, V, K]");
  }
  if (output.has_value()) {
    cuda_contig(*output, "output");
    dtype(*output, "output", at::kBFloat16);
    same_device(q, *output, "output");
    TORCH_CHECK_VALUE(output->sizes() == at::IntArrayRef({B, T, Hv, kHead}),
                      "output must have shape [B, T, HV, V]");
  } else {
    output = at::empty_like(v);
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int flags = (qk_l2norm ? GDN_POOL_QK_L2NORM : 0) | (no_state_update ? GDN_POOL_NO_STATE_UPDATE : 0);
  check_rc(gdn_decode_pool(q.data_ptr(), k.data_ptr(), v.data_ptr(), A_log.data_ptr<float>(), a.data_ptr(),
                           dt_bias.data_ptr<float>(), b.data_ptr(), static_cast<float>(scale),
                           state_pool.data_ptr(),
                           state_pool.scalar_type() == at::kBFloat16 ? GDN_STATE_BF16 : GDN_STATE_F32, P,
                           in_slots.data_ptr<int32_t>(),
                           out_slots.has_value() ? out_slots->data_ptr<int32_t>() : nullptr,
                           intermediate.has_value() ? intermediate->data_ptr() : nullptr, flags,
                           output->data_ptr(), B, T, Hq, Hk, Hv, kHead, stream),
           "gdn_decode_pool");
  return *output;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch-tensor binding of the gdn_b200 C ABI";
  m.def("decode", &decode, "GDN decode (C ABI gdn_decode)", py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("state"), py::arg("A_log"), py::arg("a"), py::arg("dt_bias"), py::arg("b"),
        py::arg("scale"), py::arg("output") = py::none(), py::arg("new_state") = py::none());
  m.def("prefill", &prefill,
        "GDN prefill (C ABI gdn_prefill_ex / gdn_prefill_segmented)", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("state"), py::arg("A_log"), py::arg("a"), py::arg("dt_bias"),
        py::arg("b"), py::arg("cu_seqlens"), py::arg("scale"), py::arg("output") = py::none(),
        py::arg("new_state") = py::none(), py::arg("path") = 0, py::arg("qk_l2norm") = false,
        py::arg("segments") = 0);
  m.def("decode_pool", &decode_pool, "pooled multi-token GDN decode (C ABI gdn_decode_pool)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("A_log"), py::arg("a"), py::arg("dt_bias"),
        py::arg("b"), py::arg("scale"), py::arg("state_pool"), py::arg("in_slots"),
        py::arg("out_slots") = py::none(), py::arg("intermediate") = py::none(),
        py::arg("qk_l2norm") = false, py::arg("no_state_update") = false,
        py::arg("output") = py::none());
}
