// sv_noalloc.cu -- sv_beam_step_noalloc: the beam step for callers that cannot
// allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocating routine) for the beam
// step's workspace: a host application that owns the GPU's memory through its own
// pool and does not let plugins allocate behind its back, or a generation loop that
// must not allocate while a step is running.  This entry point takes the workspace
// from a fixed array in device memory that the library itself declares, so the
// caller passes only inputs and outputs.
//
// The array lives for as long as the library is loaded: every GPU that loads the
// library holds kNoAllocScratchBytes (8 MiB) of it until the process exits.  All
// calls share it, so calls that overlap on the GPU (different streams, different
// host threads) race and must be serialised by the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/starvector_sampling.h"
#include "sv_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

// The shared scratch.  In host code this name is only a stand-in for the device
// array: its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) unsigned char g_beam_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of the scratch on the current device, looked up once per device
// and kept for the life of the process (it does not survive a device reset).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_beam_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int sv_beam_step_noalloc(const void* logits, int32_t logits_dtype, int32_t beams, int32_t vocab,
                                    int64_t logits_row_stride, const void* history, int32_t history_kind,
                                    int64_t history_row_stride, const int32_t* history_len, int32_t history_cols,
                                    const float* running_scores, const float* uniforms, int32_t num_picks,
                                    double temperature, double top_p, int32_t top_k, int32_t keep,
                                    double repetition_penalty, int64_t* out_picks, float* out_pick_scores,
                                    int32_t* out_num_picks, int32_t* out_status, int32_t* out_kept_count,
                                    int32_t* out_kept_idx, float* out_kept_logprob, float* out_kept_prob,
                                    int32_t out_capacity, float* out_dense_logprob, int64_t dense_row_stride,
                                    int32_t flags, void* stream) {
  const size_t need = sv_beam_workspace_bytes(beams, vocab);
  if (need == 0) return SV_E_SHAPE;
  if (need > kNoAllocScratchBytes) return SV_E_NOALLOC_LIMIT;
  void* ws = nullptr;
  if (scratch_address(&ws) != cudaSuccess) return SV_E_CUDA;
  // The previous call leaves its data behind; the merge counter and the per-beam
  // status/count header must start at zero.
  if (cudaMemsetAsync(ws, 0, sizeof(sv::BeamWsHeader), static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return SV_E_CUDA;
  return sv_beam_step(logits, logits_dtype, beams, vocab, logits_row_stride, history, history_kind,
                      history_row_stride, history_len, history_cols, running_scores, uniforms, num_picks,
                      temperature, top_p, top_k, keep, repetition_penalty, out_picks, out_pick_scores,
                      out_num_picks, out_status, out_kept_count, out_kept_idx, out_kept_logprob, out_kept_prob,
                      out_capacity, out_dense_logprob, dense_row_stride, ws, kNoAllocScratchBytes, flags, stream);
}
