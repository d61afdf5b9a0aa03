// sv_torch.cpp -- the thin PyTorch C++ extension over the C ABI
// (include/starvector_sampling.h).
//
// Each function takes torch tensors, checks them (device, dtype, sizes) with
// TORCH_CHECK, calls the C entry point on the tensors' current CUDA stream and
// returns its code (0 or a negative SV_E_*; ops.py turns codes into the same
// exceptions as before).  Shapes and the history form are decided by the Python
// wrappers (ops.py), which pass the same sizes and strides as the C signatures;
// nothing here synchronises or allocates.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdint>
#include <optional>

#include "../../include/starvector_sampling.h"

namespace {

using OptT = std::optional<at::Tensor>;

void on_device(const at::Tensor& t, const at::Device& dev, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (the B200 sampling kernels have no CPU path)");
  TORCH_CHECK(t.device() == dev, name, " must be on ", dev, ", not ", t.device());
}

template <typename T>
T* ptr(const at::Tensor& t, const at::Device& dev, const char* name, at::ScalarType st, int64_t min_numel = 1) {
  on_device(t, dev, name);
  TORCH_CHECK(t.scalar_type() == st, name, " must be ", st, ", not ", t.scalar_type());
  TORCH_CHECK(t.numel() >= min_numel, name, " holds ", t.numel(), " elements, needs ", min_numel);
  return reinterpret_cast<T*>(t.data_ptr());
}

template <typename T>
T* optptr(const OptT& t, const at::Device& dev, const char* name, at::ScalarType st, int64_t min_numel = 1) {
  return t.has_value() ? ptr<T>(*t, dev, name, st, min_numel) : nullptr;
}

void* raw(const OptT& t, const at::Device& dev, const char* name) {
  if (!t.has_value()) return nullptr;
  on_device(*t, dev, name);
  return t->data_ptr();
}

int32_t logit_code(const at::Tensor& x) {
  switch (x.scalar_type()) {
    case at::kFloat: return SV_F32;
    case at::kHalf: return SV_F16;
    case at::kBFloat16: return SV_BF16;
    default: TORCH_CHECK(false, "logits must be float32, float16 or bfloat16, not ", x.scalar_type());
  }
  return -1;
}

void* stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// sv_sample_step (runtime_shared.py:194-202).
int sample_step(const at::Tensor& logits, int64_t rows, int64_t vocab, int64_t row_stride, const OptT& history,
                 int64_t history_kind, int64_t history_row_stride, const OptT& history_len, int64_t history_cols,
                 const at::Tensor& uniforms, double temperature, double top_p, int64_t top_k, int64_t keep,
                 double repetition_penalty, const at::Tensor& out_token, const OptT& out_count, const OptT& out_idx,
                 const OptT& out_prob, const OptT& out_score, int64_t out_capacity, const OptT& out_dense,
                 int64_t dense_mode, int64_t dense_row_stride, const at::Tensor& out_status, const OptT& seen_update,
                 int64_t seen_update_row_stride, int64_t flags) {
  const at::Device dev = logits.device();
  on_device(logits, dev, "logits");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = sv_sample_step(
      logits.data_ptr(), logit_code(logits), (int32_t)rows, (int32_t)vocab, row_stride, raw(history, dev, "history"),
      (int32_t)history_kind, history_row_stride, optptr<int32_t>(history_len, dev, "history_len", at::kInt, rows),
      (int32_t)history_cols, ptr<float>(uniforms, dev, "uniforms", at::kFloat, rows), temperature, top_p,
      (int32_t)top_k, (int32_t)keep, repetition_penalty, ptr<int64_t>(out_token, dev, "token", at::kLong, rows),
      optptr<int32_t>(out_count, dev, "count", at::kInt, rows),
      optptr<int32_t>(out_idx, dev, "idx", at::kInt, rows * out_capacity),
      optptr<float>(out_prob, dev, "prob", at::kFloat, rows * out_capacity),
      optptr<float>(out_score, dev, "score", at::kFloat, rows * out_capacity), (int32_t)out_capacity,
      optptr<float>(out_dense, dev, "dense", at::kFloat, rows * vocab), (int32_t)dense_mode, dense_row_stride,
      ptr<int32_t>(out_status, dev, "status", at::kInt, rows),
      optptr<uint32_t>(seen_update, dev, "update_seen_bits", at::kInt), seen_update_row_stride, (int32_t)flags,
      stream_of(logits));
  return rc;
}

// sv_beam_step (runtime_shared.py:230-237).
int beam_step(const at::Tensor& logits, int64_t beams, int64_t vocab, int64_t row_stride, const OptT& history,
               int64_t history_kind, int64_t history_row_stride, const OptT& history_len, int64_t history_cols,
               const at::Tensor& running_scores, const at::Tensor& uniforms, int64_t num_picks, double temperature,
               double top_p, int64_t top_k, int64_t keep, double repetition_penalty, const at::Tensor& out_picks,
               const at::Tensor& out_pick_scores, const at::Tensor& out_num_picks, const at::Tensor& out_status,
               const OptT& out_kept_count, const OptT& out_kept_idx, const OptT& out_kept_logprob,
               const OptT& out_kept_prob, int64_t out_capacity, const OptT& out_dense_logprob,
               int64_t dense_row_stride, const at::Tensor& workspace, int64_t flags) {
  const at::Device dev = logits.device();
  on_device(logits, dev, "logits");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = sv_beam_step(
      logits.data_ptr(), logit_code(logits), (int32_t)beams, (int32_t)vocab, row_stride,
      raw(history, dev, "history"), (int32_t)history_kind, history_row_stride,
      optptr<int32_t>(history_len, dev, "history_len", at::kInt, beams), (int32_t)history_cols,
      ptr<float>(running_scores, dev, "running_scores", at::kFloat, beams),
      ptr<float>(uniforms, dev, "uniforms", at::kFloat, num_picks), (int32_t)num_picks, temperature, top_p,
      (int32_t)top_k, (int32_t)keep, repetition_penalty, ptr<int64_t>(out_picks, dev, "picks", at::kLong, num_picks),
      ptr<float>(out_pick_scores, dev, "scores", at::kFloat, num_picks),
      ptr<int32_t>(out_num_picks, dev, "n", at::kInt), ptr<int32_t>(out_status, dev, "status", at::kInt),
      optptr<int32_t>(out_kept_count, dev, "kept_count", at::kInt, beams),
      optptr<int32_t>(out_kept_idx, dev, "kept_idx", at::kInt, beams * out_capacity),
      optptr<float>(out_kept_logprob, dev, "kept_logprob", at::kFloat, beams * out_capacity),
      optptr<float>(out_kept_prob, dev, "kept_prob", at::kFloat, beams * out_capacity), (int32_t)out_capacity,
      optptr<float>(out_dense_logprob, dev, "dense_logprob", at::kFloat, beams * vocab), dense_row_stride,
      ptr<uint8_t>(workspace, dev, "workspace", at::kByte), (size_t)workspace.numel(), (int32_t)flags,
      stream_of(logits));
  return rc;
}

// sv_beam_advance (runtime_shared.py:237-259).
int beam_advance(const at::Tensor& picks, const at::Tensor& pick_scores, const at::Tensor& n_picks,
                  const at::Tensor& status, int64_t beams, int64_t vocab, int64_t step, bool last,
                  const OptT& stop_ids, int64_t eos_id, const OptT& tails_in, const OptT& tails_out,
                  const at::Tensor& running_out, const at::Tensor& parents_out, const at::Tensor& tokens_out,
                  const OptT& seen_in, const OptT& seen_out, int64_t seen_stride_words, const OptT& hist_in,
                  const OptT& hist_out, int64_t hist_stride, const OptT& whash_in, const OptT& whash_out,
                  const OptT& guard_table, int64_t window) {
  const at::Device dev = picks.device();
  const c10::cuda::CUDAGuard guard(dev);
  const int64_t num_picks = picks.numel();
  const int64_t n_stop = stop_ids.has_value() ? stop_ids->numel() : 0;
  const int rc = sv_beam_advance(
      ptr<int64_t>(picks, dev, "picks", at::kLong), ptr<float>(pick_scores, dev, "scores", at::kFloat, num_picks),
      ptr<int32_t>(n_picks, dev, "n", at::kInt), ptr<int32_t>(status, dev, "status", at::kInt), (int32_t)beams,
      (int32_t)vocab, (int32_t)num_picks, (int32_t)step, last ? 1 : 0,
      n_stop ? optptr<int64_t>(stop_ids, dev, "stop_ids", at::kLong) : nullptr, (int32_t)n_stop, eos_id,
      n_stop ? optptr<int64_t>(tails_in, dev, "tails_in", at::kLong, beams * n_stop) : nullptr,
      n_stop ? optptr<int64_t>(tails_out, dev, "tails_out", at::kLong, beams * n_stop) : nullptr,
      ptr<float>(running_out, dev, "running_out", at::kFloat, beams),
      ptr<int64_t>(parents_out, dev, "parents_out", at::kLong, beams),
      ptr<int64_t>(tokens_out, dev, "tokens_out", at::kLong, beams),
      optptr<uint32_t>(seen_in, dev, "seen_in", at::kInt), optptr<uint32_t>(seen_out, dev, "seen_out", at::kInt),
      seen_stride_words, optptr<int32_t>(hist_in, dev, "hist_in", at::kInt),
      optptr<int32_t>(hist_out, dev, "hist_out", at::kInt), hist_stride,
      optptr<uint32_t>(whash_in, dev, "whash_in", at::kInt, beams),
      optptr<uint32_t>(whash_out, dev, "whash_out", at::kInt, beams),
      optptr<unsigned long long>(guard_table, dev, "guard_table", at::kLong),
      guard_table.has_value() ? guard_table->numel() : 0, (int32_t)window, stream_of(picks));
  return rc;
}

// sv_kv_reorder (runtime_shared.py:388-394).
int kv_reorder(const at::Tensor& keys, const OptT& values, int64_t layers, int64_t beams, int64_t heads,
                int64_t length, int64_t head_dim, int64_t stride_layer, int64_t stride_beam, int64_t stride_head,
                int64_t stride_slot, const at::Tensor& parents, const OptT& out_status) {
  const at::Device dev = keys.device();
  on_device(keys, dev, "keys");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = sv_kv_reorder(keys.data_ptr(), raw(values, dev, "values"), (int32_t)keys.element_size(),
                               (int32_t)layers, (int32_t)beams, (int32_t)heads, length, (int32_t)head_dim,
                               stride_layer, stride_beam, stride_head, stride_slot,
                               ptr<int64_t>(parents, dev, "parents", at::kLong, beams),
                               optptr<int32_t>(out_status, dev, "status", at::kInt), stream_of(keys));
  return rc;
}

// sv_loop_guard (runtime_shared.py:156-167).
int loop_guard(const at::Tensor& tokens, int64_t rows, int64_t row_stride, const at::Tensor& lengths, int64_t window,
                int64_t repeats, const at::Tensor& out_verdict) {
  const at::Device dev = tokens.device();
  on_device(tokens, dev, "tokens");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = sv_loop_guard(tokens.data_ptr(), (int32_t)tokens.element_size(), (int32_t)rows, row_stride,
                               ptr<int32_t>(lengths, dev, "lengths", at::kInt, rows), (int32_t)window,
                               (int32_t)repeats, ptr<uint8_t>(out_verdict, dev, "verdict", at::kByte, rows),
                               stream_of(tokens));
  return rc;
}

// sv_loop_guard_incremental (runtime_shared.py:156-167, :207, :254).
int loop_guard_incremental(const at::Tensor& table, const at::Tensor& tokens, int64_t insert_from, int64_t length,
                            int64_t window, int64_t repeats, const at::Tensor& out_verdict, const OptT& out_status) {
  const at::Device dev = tokens.device();
  on_device(tokens, dev, "tokens");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = sv_loop_guard_incremental(
      ptr<unsigned long long>(table, dev, "table", at::kLong), table.numel(), tokens.data_ptr(),
      (int32_t)tokens.element_size(), insert_from, length, (int32_t)window, (int32_t)repeats,
      ptr<uint8_t>(out_verdict, dev, "verdict", at::kByte), optptr<int32_t>(out_status, dev, "status", at::kInt),
      stream_of(tokens));
  return rc;
}

}  // namespace

PYBIND11_MODULE(sv_torch, m) {
  m.doc() = "Thin PyTorch extension over the StarVector B200 sampling C ABI (include/starvector_sampling.h)";
  m.def("abi_version", &sv_abi_version);
  m.def("sample_step", &sample_step);
  m.def("beam_step", &beam_step);
  m.def("beam_advance", &beam_advance);
  m.def("kv_reorder", &kv_reorder);
  m.def("loop_guard", &loop_guard);
  m.def("loop_guard_incremental", &loop_guard_incremental);
}
