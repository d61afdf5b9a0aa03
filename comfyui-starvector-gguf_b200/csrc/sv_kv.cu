// sv_kv.cu -- the beam step's KV-cache reorder (runtime_shared.py:388-394).
//
// After a beam step each beam row r continues the sequence of beam parents[r]:
// the reference copies, for every row whose parent changed, the parent's cached
// keys and values over the first `length` slots (keys[:, rows, ..., :length, :] =
// keys[:, sources, ..., :length, :], advanced indexing: the sources are read before
// any row is written).  Here the parents come from device memory (no host sync) and
// one thread owns a 16-byte vector position of a (layer, head, slot) across all
// changed rows: it loads every changed row's source vector first and stores them
// after, so any permutation (swaps, several rows taking one parent) is copied as the
// reference's gather-then-scatter.  Rows whose parent is themselves are not touched.
// The loads are plain global loads (not the read-only path): the same addresses are
// written by this thread afterwards, and the compiler must keep that order.
// HBM-bound: 2 x (changed rows) x layers x heads x length x head_dim x element bytes
// per cache tensor.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/starvector_sampling.h"

namespace {

constexpr int kMaxKvBeams = 8;  // the node's num_beams maximum (nodes.py:128)
constexpr int KNT = 256;
constexpr int kVecRegs = 8;  // 16-byte vectors a thread holds between its loads and stores

struct KvArgs {
  unsigned char* cache[2];  // keys, values (values may be null)
  int64_t s_layer, s_beam, s_head, s_slot;  // strides in bytes
  int beams, heads;
  int64_t length;
  int dv;  // 16-byte vectors per head_dim row
  const int64_t* parents;
  int32_t* out_status;
};

// Copies with at most C changed rows: each thread moves U = kVecRegs / C vector
// positions per pass, all loads of a pass issued before its stores.
template <int C>
__device__ __forceinline__ void reorder_rows(const KvArgs a, unsigned char* base, const int* dst, const int* src,
                                             int nc) {
  constexpr int U = C >= kVecRegs ? 1 : kVecRegs / C;
  const int n = (int)a.length * a.dv;  // vectors of one (layer, head, beam); < 2^31 (host check)
  const int step = gridDim.x * KNT;
  for (int64_t i0 = blockIdx.x * KNT + threadIdx.x; i0 < n; i0 += (int64_t)step * U) {
    uint4 v[U][C];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + (int64_t)u * step;
      const int iv = (int)i;  // i < n < 2^30 wherever it is used
      const int64_t off = (int64_t)(iv / a.dv) * a.s_slot + (iv % a.dv) * 16;
#pragma unroll
      for (int c = 0; c < C; ++c)
        if (c < nc && i < n) v[u][c] = *reinterpret_cast<const uint4*>(base + src[c] * a.s_beam + off);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + (int64_t)u * step;
      const int iv = (int)i;  // i < n < 2^30 wherever it is used
      const int64_t off = (int64_t)(iv / a.dv) * a.s_slot + (iv % a.dv) * 16;
#pragma unroll
      for (int c = 0; c < C; ++c)
        if (c < nc && i < n) *reinterpret_cast<uint4*>(base + dst[c] * a.s_beam + off) = v[u][c];
    }
  }
}

__global__ void __launch_bounds__(KNT) kv_reorder_kernel(const KvArgs a) {
  __shared__ int dst[kMaxKvBeams], src[kMaxKvBeams];
  __shared__ int nchanged;
  if (threadIdx.x < 32) {
    const int r = threadIdx.x;
    const bool row = r < a.beams;
    const int64_t p = row ? a.parents[r] : r;
    const bool ok = row && p >= 0 && p < a.beams;  // an invalid parent leaves its row as it is
    const bool chg = ok && p != r;
    const unsigned m = __ballot_sync(0xffffffffu, chg);
    const unsigned bad = __ballot_sync(0xffffffffu, row && !ok);
    if (chg) {
      const int pos = __popc(m & ((1u << r) - 1u));
      dst[pos] = r;
      src[pos] = (int)p;
    }
    if (r == 0) {
      nchanged = __popc(m);
      if (a.out_status && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) *a.out_status = bad != 0u;
    }
  }
  __syncthreads();
  const int nc = nchanged;
  if (!nc) return;
  const int lh = blockIdx.y;  // layer * heads + head
  const int64_t l = lh / a.heads, h = lh % a.heads;
  unsigned char* base = (blockIdx.z ? a.cache[1] : a.cache[0]) + l * a.s_layer + h * a.s_head;
  if (nc <= 1)
    reorder_rows<1>(a, base, dst, src, nc);
  else if (nc <= 2)
    reorder_rows<2>(a, base, dst, src, nc);
  else if (nc <= 4)
    reorder_rows<4>(a, base, dst, src, nc);
  else
    reorder_rows<8>(a, base, dst, src, nc);
}

}  // namespace

// See include/starvector_sampling.h.
extern "C" int sv_kv_reorder(void* keys, void* values, int32_t elem_bytes, int32_t layers, int32_t beams,
                             int32_t heads, int64_t length, int32_t head_dim, int64_t stride_layer,
                             int64_t stride_beam, int64_t stride_head, int64_t stride_slot, const int64_t* parents,
                             int32_t* out_status, void* stream) {
  if (!keys || !parents) return SV_E_ARG;
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4) return SV_E_DTYPE;
  if (layers < 1 || beams < 1 || beams > kMaxKvBeams || heads < 1 || head_dim < 1 || length < 0) return SV_E_SHAPE;
  if ((int64_t)layers * heads > 65535) return SV_E_SHAPE;
  const int64_t row = (int64_t)head_dim * elem_bytes;
  const int64_t sb[4] = {stride_layer * elem_bytes, stride_beam * elem_bytes, stride_head * elem_bytes,
                         stride_slot * elem_bytes};
  if (row % 16) return SV_E_ALIGN;
  for (int k = 0; k < 4; ++k)
    if (sb[k] % 16 || sb[k] < 0) return SV_E_ALIGN;
  if (reinterpret_cast<uintptr_t>(keys) % 16 || reinterpret_cast<uintptr_t>(values) % 16) return SV_E_ALIGN;
  if (length * (row / 16) >= (int64_t)1 << 30) return SV_E_SHAPE;
  if (length == 0) return SV_OK;
  KvArgs a;
  a.cache[0] = static_cast<unsigned char*>(keys);
  a.cache[1] = static_cast<unsigned char*>(values);
  a.s_layer = sb[0];
  a.s_beam = sb[1];
  a.s_head = sb[2];
  a.s_slot = sb[3];
  a.beams = beams;
  a.heads = heads;
  a.length = length;
  a.dv = (int)(row / 16);
  a.parents = parents;
  a.out_status = out_status;
  const int64_t n = length * a.dv;
  int64_t gx = (n + KNT - 1) / KNT;
  // About 8 blocks per SM over the whole grid, whatever layers * heads is; each
  // thread keeps kVecRegs vectors in flight whatever the number of changed rows.
  const int64_t lhz = (int64_t)layers * heads * (values ? 2 : 1);
  const int64_t want = (8 * 148 + lhz - 1) / lhz;
  if (gx > want) gx = want > 0 ? want : 1;
  const dim3 grid((unsigned)gx, (unsigned)(layers * heads), values ? 2u : 1u);
  kv_reorder_kernel<<<grid, KNT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}
