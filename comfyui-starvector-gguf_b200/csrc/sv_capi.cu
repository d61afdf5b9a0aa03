// sv_capi.cu -- the extern "C" entry points of include/starvector_sampling.h.
//
// Validates arguments (mirroring the reference's ValueError conditions,
// runtime_shared.py:277-300, plus the shape limits of the kernels), chooses the
// cluster split of each row and launches.  No allocation, no synchronisation.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstdint>

#include "../../include/starvector_sampling.h"
#include "sv_internal.h"

namespace sv {
cudaError_t launch_loop_guard(const void* tokens, int token_bytes, int rows, int64_t stride, const int32_t* lengths,
                              int window, int repeats, uint8_t* verdict, cudaStream_t stream);
int loop_guard_max_window();
cudaError_t launch_penalize(const void* x, int dtype, int64_t xstride, int rows, int64_t V, int hist_kind,
                            const void* hist, int64_t hstride, float rp, float* out, int64_t ostride,
                            cudaStream_t stream);
cudaError_t launch_seen_update(uint32_t* bits, int rows, int64_t stride, const int64_t* tokens, int64_t vocab,
                               cudaStream_t stream);
cudaError_t launch_seen_reorder(const uint32_t* src, uint32_t* dst, int beams, int64_t words, int64_t stride,
                                const int64_t* parents, const int64_t* tokens, int64_t vocab, cudaStream_t stream);
}  // namespace sv

using namespace sv;

namespace {

constexpr int64_t kMaxVocab = 524288;
constexpr size_t kSmemLimit = 226 * 1024;  // leaves room for the merge's static shared memory
constexpr int kSMs = 148;

int esize(int dtype) { return dtype == DT_F32 ? 4 : 2; }

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Region A of a CTA: the staged slice + its seen mask, or the leader's work arrays
// (16 KB), or the general path's bitmap of the whole row.
size_t region_a_bytes(int64_t V, int es, int slice_len) {
  size_t stage = round_up((size_t)slice_len * es + 32, 128) + round_up((size_t)slice_len + 64, 128);
  size_t leader = 16 * (size_t)kCandCap;
  size_t general = round_up((size_t)(V + 31) / 32 * 4, 128) + 4096;
  size_t a = stage > leader ? stage : leader;
  return a > general ? a : general;
}

// Tuning override of the cluster split (CTAs per row), read once: SV_ROW_SPLIT=1..16.
int split_override() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("SV_ROW_SPLIT");
    int s = e ? std::atoi(e) : 0;
    v = (s == 1 || s == 2 || s == 4 || s == 8 || s == 16) ? s : 0;
  }
  return v;
}

// Rows from which sv_sample_step prefers the streaming kernel; tuning override
// SV_STREAM_MIN_ROWS, read once.
int stream_min_rows() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("SV_STREAM_MIN_ROWS");
    v = e ? std::atoi(e) : 64;
    if (v < 1) v = 1;
  }
  return v;
}

// Cluster split: slices of at most 48 KB; small batches spread over more SMs.
void choose_layout(int64_t V, int es, int rows, int32_t* S_out, int32_t* slice_out, size_t* smem_out) {
  int S = 1;
  while (S < kMaxCluster && V * es / S > 48 * 1024) S <<= 1;
  while (S < kMaxCluster && (int64_t)rows * S < kSMs && V / (2 * S) >= 1536) S <<= 1;
  if (split_override()) S = split_override();
  int32_t slice = 0;
  for (;;) {
    slice = (int32_t)round_up((size_t)((V + S - 1) / S), 16);
    if (S == 1 || (int64_t)(S - 1) * slice < V) break;
    S >>= 1;
  }
  size_t smem = shared_static_bytes() + region_a_bytes(V, es, slice);
  while (smem > kSmemLimit && S < kMaxCluster) {
    S <<= 1;
    slice = (int32_t)round_up((size_t)((V + S - 1) / S), 16);
    smem = shared_static_bytes() + region_a_bytes(V, es, slice);
  }
  *S_out = S;
  *slice_out = slice;
  *smem_out = smem;
}

int check_common(const void* logits, int32_t dtype, int32_t rows, int32_t vocab, int64_t stride, const void* history,
                 int32_t hist_kind, int64_t hist_stride, int32_t hist_cols, double temperature, double top_p,
                 int32_t top_k, int32_t keep, double rp) {
  if (!logits) return SV_E_ARG;
  if (dtype != DT_F32 && dtype != DT_F16 && dtype != DT_BF16) return SV_E_DTYPE;
  if (rows < 1 || vocab < 1 || vocab > kMaxVocab || stride < 0) return SV_E_SHAPE;
  if (stride > 0 && stride < vocab) return SV_E_SHAPE;
  if (reinterpret_cast<uintptr_t>(logits) % esize(dtype)) return SV_E_ALIGN;
  if (hist_kind < HIST_NONE || hist_kind > HIST_BITS32) return SV_E_DTYPE;
  if (hist_kind != HIST_NONE) {
    if (!history || hist_stride < 0) return SV_E_ARG;
    if ((hist_kind == HIST_IDS32 || hist_kind == HIST_IDS64) && hist_cols < 0) return SV_E_SHAPE;
    const int hb = hist_kind == HIST_IDS64 ? 8 : (hist_kind == HIST_MASK8 ? 1 : 4);
    if (reinterpret_cast<uintptr_t>(history) % hb) return SV_E_ALIGN;
  }
  if (!(temperature > 0.0) || !std::isfinite(temperature)) return SV_E_RANGE;
  if (!(top_p > 0.0 && top_p <= 1.0)) return SV_E_RANGE;
  if (!(rp > 0.0) || !std::isfinite(rp)) return SV_E_RANGE;
  if (top_k < 1 || top_k > kMaxTopK || keep < 1 || keep > kMaxTopK) return SV_E_RANGE;
  const int kk = top_k > keep ? top_k : keep;
  if (kk > vocab) return SV_E_RANGE;
  return SV_OK;
}

void fill_common(RowArgs& a, const void* logits, int32_t dtype, int32_t rows, int32_t vocab, int64_t stride,
                 const void* history, int32_t hist_kind, int64_t hist_stride, const int32_t* hist_len,
                 int32_t hist_cols, double temperature, double top_p, int32_t top_k, int32_t keep, double rp) {
  a.logits = logits;
  a.dtype = dtype;
  a.rows = rows;
  a.vocab = vocab;
  a.row_stride = stride;
  a.hist = history;
  a.hist_kind = history ? hist_kind : HIST_NONE;
  a.hist_stride = hist_stride;
  a.hist_len = hist_len;
  a.hist_cols = hist_cols;
  // torch casts a Python float scalar to the tensor's dtype (float32).
  a.temperature = (float)temperature;
  a.rep_penalty = (float)rp;
  a.pthr = top_p < 1.0 ? (float)(1.0 - top_p) : 0.0f;
  a.kk = top_k > keep ? top_k : keep;
  a.keep = keep;
}

}  // namespace

extern "C" {

int sv_sample_step(const void* logits, int32_t logits_dtype, int32_t rows, int32_t vocab, int64_t logits_row_stride,
                   const void* history, int32_t history_kind, int64_t history_row_stride,
                   const int32_t* history_len, int32_t history_cols, const float* uniforms, double temperature,
                   double top_p, int32_t top_k, int32_t keep, double repetition_penalty, int64_t* out_token,
                   int32_t* out_count, int32_t* out_idx, float* out_prob, float* out_score, int32_t out_capacity,
                   float* out_dense, int32_t dense_mode, int64_t dense_row_stride, int32_t* out_status,
                   uint32_t* seen_bits_update, int64_t seen_bits_row_stride, int32_t flags, void* stream) {
  int rc = check_common(logits, logits_dtype, rows, vocab, logits_row_stride, history, history_kind,
                        history_row_stride, history_cols, temperature, top_p, top_k, keep, repetition_penalty);
  if (rc) return rc;
  if (!uniforms || !out_token) return SV_E_ARG;
  if (out_capacity < 0) return SV_E_SHAPE;
  if (dense_mode < DENSE_NONE || dense_mode > DENSE_PROBS) return SV_E_DTYPE;
  if (dense_mode != DENSE_NONE && (!out_dense || dense_row_stride < vocab)) return SV_E_ARG;
  if (seen_bits_update && seen_bits_row_stride < (vocab + 31) / 32) return SV_E_SHAPE;
  RowArgs a = {};
  fill_common(a, logits, logits_dtype, rows, vocab, logits_row_stride, history, history_kind, history_row_stride,
              history_len, history_cols, temperature, top_p, top_k, keep, repetition_penalty);
  a.mode = MODE_SAMPLE;
  a.uniforms = uniforms;
  a.out_token = out_token;
  a.out_count = out_count;
  a.out_idx = out_idx;
  a.out_prob = out_prob;
  a.out_score = out_score;
  a.out_cap = out_capacity;
  a.out_dense = dense_mode != DENSE_NONE ? out_dense : nullptr;
  a.dense_mode = dense_mode;
  a.dense_stride = dense_row_stride;
  a.out_status = out_status;
  a.seen_bits = seen_bits_update;
  a.seen_bits_stride = seen_bits_row_stride;
  a.force_slow = (flags & SV_FLAG_FORCE_GENERAL) ? 1 : 0;
  a.wait_test = (flags & SV_FLAG_TEST_WAIT_TIMEOUT) ? 1 : 0;
  // Path: the streaming kernel for many rows when the row's seen mask fits a CTA.
  const size_t ssmem = stream_smem_bytes(vocab);
  bool use_stream = ssmem > 0 && rows >= stream_min_rows();
  if (flags & SV_FLAG_CLUSTER) use_stream = false;
  if ((flags & SV_FLAG_STREAM) && ssmem > 0) use_stream = true;
  cudaError_t e;
  if (use_stream) {
    e = launch_stream(a, ssmem, static_cast<cudaStream_t>(stream));
  } else {
    size_t smem;
    choose_layout(vocab, esize(logits_dtype), rows, &a.S, &a.slice_len, &smem);
    a.region_a = (uint32_t)(smem - shared_static_bytes());
    if (smem > kSmemLimit) return SV_E_SHAPE;
    e = launch_rows(a, smem, static_cast<cudaStream_t>(stream));
  }
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

size_t sv_beam_workspace_bytes(int32_t beams, int32_t vocab) {
  if (beams < 1 || vocab < 1) return 0;
  return sizeof(BeamWsHeader) + (size_t)beams * (size_t)vocab * 16;
}

int sv_beam_step(const void* logits, int32_t logits_dtype, int32_t beams, int32_t vocab, int64_t logits_row_stride,
                 const void* history, int32_t history_kind, int64_t history_row_stride, const int32_t* history_len,
                 int32_t history_cols, const float* running_scores, const float* uniforms, int32_t num_picks,
                 double temperature, double top_p, int32_t top_k, int32_t keep, double repetition_penalty,
                 int64_t* out_picks, float* out_pick_scores, int32_t* out_num_picks, int32_t* out_status,
                 int32_t* out_kept_count, int32_t* out_kept_idx, float* out_kept_logprob, float* out_kept_prob,
                 int32_t out_capacity, float* out_dense_logprob, int64_t dense_row_stride, void* workspace,
                 size_t workspace_bytes, int32_t flags, void* stream) {
  int rc = check_common(logits, logits_dtype, beams, vocab, logits_row_stride, history, history_kind,
                        history_row_stride, history_cols, temperature, top_p, top_k, keep, repetition_penalty);
  if (rc) return rc;
  if (beams > kMaxBeams) return SV_E_SHAPE;
  if (num_picks < 1 || num_picks > 2 * kMaxBeams) return SV_E_SHAPE;
  if (!running_scores || !uniforms || !out_picks || !out_pick_scores || !out_num_picks || !out_status)
    return SV_E_ARG;
  if (out_capacity < 0) return SV_E_SHAPE;
  if (out_dense_logprob && dense_row_stride < vocab) return SV_E_SHAPE;
  if (!workspace || workspace_bytes < sv_beam_workspace_bytes(beams, vocab)) return SV_E_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return SV_E_ALIGN;
  RowArgs a = {};
  fill_common(a, logits, logits_dtype, beams, vocab, logits_row_stride, history, history_kind, history_row_stride,
              history_len, history_cols, temperature, top_p, top_k, keep, repetition_penalty);
  a.mode = MODE_BEAM;
  a.running = running_scores;
  a.uniforms = uniforms;
  a.npick = num_picks;
  a.out_picks = out_picks;
  a.out_pick_scores = out_pick_scores;
  a.out_npicks = out_num_picks;
  a.out_status = out_status;
  a.out_count = out_kept_count;
  a.out_idx = out_kept_idx;
  a.out_score = out_kept_logprob;
  a.out_prob = out_kept_prob;
  a.out_cap = out_capacity;
  a.out_dense = out_dense_logprob;
  a.dense_mode = out_dense_logprob ? DENSE_SCORES : DENSE_NONE;
  a.dense_stride = dense_row_stride;
  a.ws = static_cast<unsigned char*>(workspace);
  a.ws_cap = vocab;
  a.force_slow = (flags & SV_FLAG_FORCE_GENERAL) ? 1 : 0;
  size_t smem;
  choose_layout(vocab, esize(logits_dtype), beams, &a.S, &a.slice_len, &smem);
  a.region_a = (uint32_t)(smem - shared_static_bytes());
  if (smem > kSmemLimit) return SV_E_SHAPE;
  cudaError_t e = launch_rows(a, smem, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

int sv_loop_guard(const void* tokens, int32_t token_bytes, int32_t rows, int64_t row_stride, const int32_t* lengths,
                  int32_t window, int32_t repeats, uint8_t* out_verdict, void* stream) {
  if (!tokens || !lengths || !out_verdict) return SV_E_ARG;
  if (token_bytes != 4 && token_bytes != 8) return SV_E_DTYPE;
  if (rows < 1 || row_stride < 0) return SV_E_SHAPE;
  if (window < 1 || window > loop_guard_max_window() || repeats < 1) return SV_E_RANGE;
  if (reinterpret_cast<uintptr_t>(tokens) % token_bytes) return SV_E_ALIGN;
  cudaError_t e = launch_loop_guard(tokens, token_bytes, rows, row_stride, lengths, window, repeats, out_verdict,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

int sv_penalize(const void* logits, int32_t logits_dtype, int32_t rows, int32_t vocab, int64_t logits_row_stride,
                const void* history, int32_t history_kind, int64_t history_row_stride, double repetition_penalty,
                float* out, int64_t out_row_stride, void* stream) {
  if (!logits || !history || !out) return SV_E_ARG;
  if (logits_dtype != DT_F32 && logits_dtype != DT_F16 && logits_dtype != DT_BF16) return SV_E_DTYPE;
  if (history_kind != HIST_MASK8 && history_kind != HIST_BITS32) return SV_E_DTYPE;
  if (rows < 1 || vocab < 1 || logits_row_stride < 0 || out_row_stride < vocab) return SV_E_SHAPE;
  if (!(repetition_penalty > 0.0) || !std::isfinite(repetition_penalty)) return SV_E_RANGE;
  cudaError_t e = launch_penalize(logits, logits_dtype, logits_row_stride, rows, vocab, history_kind, history,
                                  history_row_stride, (float)repetition_penalty, out, out_row_stride,
                                  static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

int sv_seen_update(uint32_t* seen_bits, int32_t rows, int64_t row_stride_words, const int64_t* tokens, int32_t vocab,
                   void* stream) {
  if (!seen_bits || !tokens) return SV_E_ARG;
  if (rows < 1 || vocab < 1 || row_stride_words < (vocab + 31) / 32) return SV_E_SHAPE;
  cudaError_t e = launch_seen_update(seen_bits, rows, row_stride_words, tokens, vocab,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

int sv_seen_reorder(const uint32_t* src, uint32_t* dst, int32_t beams, int32_t vocab, int64_t row_stride_words,
                    const int64_t* parents, const int64_t* tokens, void* stream) {
  if (!src || !dst || !parents) return SV_E_ARG;
  if (beams < 1 || vocab < 1 || row_stride_words < (vocab + 31) / 32) return SV_E_SHAPE;
  const int64_t words = (vocab + 31) / 32;
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(src), d0 = reinterpret_cast<uintptr_t>(dst);
  const uintptr_t span = (uintptr_t)beams * row_stride_words * 4;
  if (s0 < d0 + span && d0 < s0 + span) return SV_E_ARG;
  cudaError_t e = launch_seen_reorder(src, dst, beams, words, row_stride_words, parents, tokens, vocab,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

const char* sv_error_string(int32_t code) {
  switch (code) {
    case SV_OK: return "ok";
    case SV_E_ARG: return "invalid argument (null pointer or inconsistent arguments)";
    case SV_E_DTYPE: return "unknown dtype, history kind or dense mode";
    case SV_E_SHAPE: return "rows, vocab, strides or capacities out of range";
    case SV_E_RANGE: return "temperature, top_p, top_k, keep or repetition_penalty out of range";
    case SV_E_ALIGN: return "pointer not aligned to its element size";
    case SV_E_WORKSPACE: return "workspace missing or too small";
    case SV_E_CUDA: return "CUDA launch failed";
    case SV_E_NOALLOC_LIMIT: return "beams x vocab exceed the fixed scratch of sv_beam_step_noalloc (8 MiB)";
    case SV_ST_NAN: return "NaN logit in row";
    case SV_ST_POSINF: return "+inf score in row";
    case SV_ST_ALLNEGINF: return "no finite logit in row";
    case SV_ST_HISTORY: return "history id outside [0, vocab)";
    case SV_ST_TIMEOUT: return "asynchronous copy wait timed out";
    case SV_ST_SHARD_OVERFLOW: return "a vocabulary slice kept more tokens than its list holds (sample unsharded)";
    case SV_ST_GUARD_FULL: return "the loop guard's window table is full";
    default: return "unknown code";
  }
}

int32_t sv_abi_version(void) { return 1; }

}  // extern "C"
