// sv_aux.cu -- small element-wise kernels around the sampling step.
//
//  * penalize_kernel: the reference's _penalize (runtime_shared.py:170-173) as a
//    dense fp32 output, for callers that use it on its own.
//  * seen_update_kernel: seen[token] = True per row (runtime_shared.py:202) on a
//    packed bitmap.
//  * seen_reorder_kernel: seen = seen[parents]; seen[b, token_b] = True
//    (runtime_shared.py:258-259) on packed bitmaps, out of place.
#include <cuda_runtime.h>

#include <cstdint>

#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

template <typename TIn>
__global__ void penalize_kernel(const TIn* __restrict__ x, int64_t xstride, int rows, int64_t V, int hist_kind,
                                const void* __restrict__ hist, int64_t hstride, float rp, float* __restrict__ out,
                                int64_t ostride) {
  const int64_t n = (int64_t)rows * V;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = k / V, i = k - r * V;
    float v = Elem<TIn>::to_f(x[r * xstride + i]);
    bool s;
    if (hist_kind == HIST_MASK8) s = reinterpret_cast<const unsigned char*>(hist)[r * hstride + i] != 0;
    else s = (reinterpret_cast<const uint32_t*>(hist)[r * hstride + (i >> 5)] >> (i & 31)) & 1u;
    out[r * ostride + i] = s ? penalize(v, rp) : v;
  }
}

__global__ void seen_update_kernel(uint32_t* bits, int rows, int64_t stride, const int64_t* __restrict__ tokens,
                                   int64_t vocab) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int64_t t = tokens[r];
  if (t >= 0 && t < vocab) atomicOr(&bits[r * stride + (t >> 5)], 1u << (t & 31));
}

__global__ void seen_reorder_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst, int beams,
                                    int64_t words, int64_t stride, const int64_t* __restrict__ parents,
                                    const int64_t* __restrict__ tokens, int64_t vocab) {
  const int b = blockIdx.y;
  const int64_t p = parents[b];
  const int64_t t = tokens ? tokens[b] : -1;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < words; w += (int64_t)gridDim.x * blockDim.x) {
    uint32_t v = (p >= 0 && p < beams) ? src[p * stride + w] : 0u;
    if (t >= 0 && t < vocab && (t >> 5) == w) v |= 1u << (t & 31);
    dst[b * stride + w] = v;
  }
}

cudaError_t launch_penalize(const void* x, int dtype, int64_t xstride, int rows, int64_t V, int hist_kind,
                            const void* hist, int64_t hstride, float rp, float* out, int64_t ostride,
                            cudaStream_t stream) {
  const int64_t n = (int64_t)rows * V;
  const int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  if (dtype == DT_F32)
    penalize_kernel<float><<<blocks, 256, 0, stream>>>(reinterpret_cast<const float*>(x), xstride, rows, V,
                                                        hist_kind, hist, hstride, rp, out, ostride);
  else if (dtype == DT_F16)
    penalize_kernel<__half><<<blocks, 256, 0, stream>>>(reinterpret_cast<const __half*>(x), xstride, rows, V,
                                                         hist_kind, hist, hstride, rp, out, ostride);
  else
    penalize_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), xstride,
                                                                rows, V, hist_kind, hist, hstride, rp, out, ostride);
  return cudaGetLastError();
}

cudaError_t launch_seen_update(uint32_t* bits, int rows, int64_t stride, const int64_t* tokens, int64_t vocab,
                               cudaStream_t stream) {
  seen_update_kernel<<<(rows + 127) / 128, 128, 0, stream>>>(bits, rows, stride, tokens, vocab);
  return cudaGetLastError();
}

cudaError_t launch_seen_reorder(const uint32_t* src, uint32_t* dst, int beams, int64_t words, int64_t stride,
                                const int64_t* parents, const int64_t* tokens, int64_t vocab, cudaStream_t stream) {
  dim3 grid((unsigned)((words + 255) / 256), (unsigned)beams);
  seen_reorder_kernel<<<grid, 256, 0, stream>>>(src, dst, beams, words, stride, parents, tokens, vocab);
  return cudaGetLastError();
}

}  // namespace sv
