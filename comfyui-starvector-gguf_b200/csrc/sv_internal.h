// sv_internal.h -- launch descriptors shared by the kernels and the C-ABI layer.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace sv {

constexpr int kThreads = 256;      // threads per CTA of the row kernel
constexpr int kGroups = 128;       // group maxima per row (lower bound of the k-th largest)
constexpr int kCandCap = 1024;     // candidate capacity of the fast path
constexpr int kMaxCluster = 16;    // CTAs per row (cluster size)
constexpr int kMaxBeams = 32;
constexpr int kChunks = 4;         // bulk copies per CTA slice
constexpr int kMaxTopK = kGroups;  // top_k (and keep) limit

enum Mode : int32_t { MODE_SAMPLE = 0, MODE_BEAM = 1 };
enum Dtype : int32_t { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };
enum HistKind : int32_t { HIST_NONE = 0, HIST_IDS32 = 1, HIST_IDS64 = 2, HIST_MASK8 = 3, HIST_BITS32 = 4 };
enum DenseMode : int32_t { DENSE_NONE = 0, DENSE_SCORES = 1, DENSE_PROBS = 2 };

// Beam workspace: header, then per beam `cap` kept (idx, value) pairs, then the
// merge weights (beams * cap u64).  The counter must be zero before a launch; the
// kernel leaves it at zero.
struct BeamWsHeader {
  uint32_t counter;
  int32_t pad[3];
  int32_t status[kMaxBeams];
  int32_t count[kMaxBeams];
};

struct RowArgs {
  // inputs
  const void* logits;
  int64_t row_stride;  // elements between rows (0 = one row broadcast)
  int32_t rows, vocab, dtype, mode;
  int32_t hist_kind;
  const void* hist;
  int64_t hist_stride;
  const int32_t* hist_len;
  int32_t hist_cols;
  const float* uniforms;  // sample: [rows]; beam: [npick]
  float temperature, rep_penalty, pthr;  // pthr = float(1 - top_p), 0 disables top-p
  int32_t kk, keep;                      // kk = max(top_k, keep)
  // per-row outputs (sample) / per-beam kept lists (beam)
  int64_t* out_token;
  int32_t* out_count;
  int32_t* out_idx;
  float* out_prob;
  float* out_score;
  int32_t out_cap;
  float* out_dense;
  int32_t dense_mode;
  int64_t dense_stride;
  int32_t* out_status;
  uint32_t* seen_bits;  // sample: set the drawn token's bit here (optional)
  int64_t seen_bits_stride;
  // beam
  const float* running;
  int32_t npick;
  int64_t* out_picks;
  float* out_pick_scores;
  int32_t* out_npicks;
  unsigned char* ws;
  int64_t ws_cap;  // kept entries per beam in the workspace (= vocab)
  // layout
  int32_t S, slice_len, force_slow;
  int32_t wait_test;  // SV_FLAG_TEST_WAIT_TIMEOUT: the history wait runs out (test hook)
  uint32_t region_a;  // bytes of the per-CTA union region
};

// Opt-in shared memory per CTA on sm_100 (227 KB).
__host__ __device__ constexpr size_t smem_limit_stream() { return 232448; }

size_t shared_static_bytes();
cudaError_t launch_rows(const RowArgs& a, size_t smem_bytes, cudaStream_t stream);
// The beam merge alone over kept lists in a.ws (a.rows beams, a.ws_cap entries each).
cudaError_t launch_beam_merge(const RowArgs& a, cudaStream_t stream);
size_t stream_smem_bytes(int64_t vocab);
cudaError_t launch_stream(const RowArgs& a, size_t smem_bytes, cudaStream_t stream);

}  // namespace sv
