// sv_shard.cu -- the merge step of the vocab-sharded sample step.
//
// With the vocabulary split across ranks, each rank runs sv_sample_step on its
// slice with top-p off (top_p = 1) and a kept-list capacity C: its kept list is
// then the slice's top-k with ties and their warped scores
// (runtime_shared.py:172-181 on the slice).  Every element at or above the row's
// k-th largest warped score is in its slice's list (fewer than k elements of the
// slice exceed it), so after an all-gather of the lists the union holds the row's
// whole top-k set.  This kernel finishes each row from that union exactly as the
// unsharded step does: the k-th largest with ties (:180-181), top-p over the
// ascending (value, index) order with exact fixed-point mass (:182-186) and the
// draw from the row's uniform (:201).
//
// Wire format (int32, one record per shard and row):
//   [0, C)      warped scores (float bits), the slice's kept tokens in index order
//   [C, 2C)     their global vocabulary indices
//   2C          kept count of the slice (may exceed C: the list was truncated)
//   2C + 1      the slice's status (SV_ST_*)
#include <cuda_runtime.h>

#include "../../include/starvector_sampling.h"
#include "sv_block.cuh"
#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

namespace {

constexpr int MNT = 256;             // threads per row
constexpr int kMergeMax = 1024;      // shards x capacity

struct MergeArgs {
  const int32_t* packed;
  int shards, rows, cap;
  const float* uniforms;
  int64_t* out_token;
  int32_t* out_count;
  int32_t* out_idx;
  float* out_prob;
  int out_cap;
  int32_t* out_status;
};

struct __align__(16) MergeShared {
  BlockScratch<MNT> bs;
  int n, err, overflow;
  __align__(16) float cv[kMergeMax];  // union; then leader_fast's P / the kept list
  int ci[kMergeMax];
  __align__(16) float fv[kMergeMax];  // candidates >= the k-th largest; then W
  int fi[kMergeMax];
  __align__(16) float sv[kMergeMax];  // ascending order; then the draw's prefix sums
  int si[kMergeMax];
};

__global__ void __launch_bounds__(MNT) merge_kernel(const MergeArgs m, const RowArgs a) {
  __shared__ MergeShared sh;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int rec = 2 * m.cap + 2;
  if (tid == 0) {
    sh.n = 0;
    sh.err = 0;
    sh.overflow = 0;
  }
  __syncthreads();
  // Union of the shards' lists.  A shard without a finite score contributes
  // nothing; any other shard error is the row's.
  for (int s = 0; s < m.shards; ++s) {
    const int32_t* r = m.packed + ((int64_t)s * m.rows + row) * rec;
    const int cnt = r[2 * m.cap], st = r[2 * m.cap + 1];
    if (st == ST_ALLNEGINF) continue;
    if (st != ST_OK) {
      if (tid == 0) sh.err |= 1 << st;
      continue;
    }
    if (cnt > m.cap && tid == 0) sh.overflow = 1;
    const int take = cnt < m.cap ? cnt : m.cap;
    __syncthreads();
    const int base = sh.n;
    for (int j = tid; j < take; j += MNT) {
      sh.cv[base + j] = __int_as_float(r[j]);
      sh.ci[base + j] = r[m.cap + j];
    }
    __syncthreads();
    if (tid == 0) sh.n = base + take;
  }
  __syncthreads();
  const int n = sh.n;
  int status = sh.err ? first_err(sh.err) : (sh.overflow ? ST_SHARD_OVERFLOW : (n == 0 ? ST_ALLNEGINF : ST_OK));
  Kept kept = {0, 0.0f, 0};
  int64_t token = -1;
  if (status == ST_OK) {
    const int mm = prefilter<MNT>(sh.bs, sh.cv, sh.ci, n, a.kk, sh.fv, sh.fi);
    int* kidx = sh.ci;
    float* kval = sh.cv;
    kept = leader_fast<MNT>(a, sh.bs, sh.fv, sh.fi, mm, sh.sv, sh.si, reinterpret_cast<uint64_t*>(sh.fv),
                            reinterpret_cast<uint64_t*>(sh.cv), kidx, kval);
    token = draw_kept<MNT>(sh.bs, kidx, kval, kept, m.uniforms[row], reinterpret_cast<uint64_t*>(sh.sv));
    const float Sf = fix_to_float(kept.tot);
    for (int j = tid; j < kept.n && j < m.out_cap; j += MNT) {
      if (m.out_idx) m.out_idx[(int64_t)row * m.out_cap + j] = kidx[j];
      if (m.out_prob) m.out_prob[(int64_t)row * m.out_cap + j] = __fdiv_rn(sv_exp(__fsub_rn(kval[j], kept.M)), Sf);
    }
  }
  if (tid == 0) {
    m.out_token[row] = status == ST_OK ? token : -1;
    if (m.out_count) m.out_count[row] = kept.n;
    if (m.out_status) m.out_status[row] = status;
  }
}

// One rank's exchange records from its slice step's outputs (one block per row).
__global__ void pack_kernel(const int32_t* count, const int32_t* status, const int32_t* idx, const float* score,
                            int cap, int offset, int32_t* out) {
  const int row = blockIdx.x;
  int32_t* r = out + (int64_t)row * (2 * cap + 2);
  for (int j = threadIdx.x; j < cap; j += blockDim.x) {
    r[j] = __float_as_int(score[(int64_t)row * cap + j]);
    r[cap + j] = idx[(int64_t)row * cap + j] + offset;
  }
  if (threadIdx.x == 0) {
    r[2 * cap] = count[row];
    r[2 * cap + 1] = status[row];
  }
}

}  // namespace

}  // namespace sv

using namespace sv;

// One rank's records [rows][2 * capacity + 2] for sv_merge_shards; see
// include/starvector_sampling.h.
extern "C" int sv_pack_slice(const int32_t* count, const int32_t* status, const int32_t* idx, const float* score,
                             int32_t rows, int32_t capacity, int32_t offset, int32_t* out_records, void* stream) {
  if (!count || !status || !idx || !score || !out_records) return SV_E_ARG;
  if (rows < 1 || capacity < 1 || capacity > kMergeMax || offset < 0) return SV_E_SHAPE;
  pack_kernel<<<rows, 64, 0, static_cast<cudaStream_t>(stream)>>>(count, status, idx, score, capacity, offset,
                                                                  out_records);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}

// Merges the all-gathered per-shard kept lists of a vocab-sharded sample step; see
// include/starvector_sampling.h.
extern "C" int sv_merge_shards(const int32_t* packed, int32_t shards, int32_t rows, int32_t capacity,
                               const float* uniforms, double top_p, int32_t top_k, int32_t keep,
                               int64_t* out_token, int32_t* out_count, int32_t* out_idx, float* out_prob,
                               int32_t out_capacity, int32_t* out_status, void* stream) {
  if (!packed || !uniforms || !out_token) return SV_E_ARG;
  if (out_capacity > 0 && !out_idx && !out_prob) return SV_E_ARG;
  if (shards < 1 || rows < 1 || capacity < 1 || (int64_t)shards * capacity > kMergeMax || out_capacity < 0)
    return SV_E_SHAPE;
  if (!(top_p > 0.0 && top_p <= 1.0)) return SV_E_RANGE;
  if (top_k < 1 || top_k > kMaxTopK || keep < 1 || keep > kMaxTopK) return SV_E_RANGE;
  const int kk = top_k > keep ? top_k : keep;
  if (kk > capacity) return SV_E_RANGE;  // a slice's top-k must fit its list
  RowArgs a = {};
  a.kk = kk;
  a.keep = keep;
  a.pthr = top_p < 1.0 ? (float)(1.0 - top_p) : 0.0f;
  MergeArgs m = {packed, shards, rows, capacity, uniforms, out_token, out_count, out_idx, out_prob, out_capacity,
                 out_status};
  merge_kernel<<<rows, MNT, 0, static_cast<cudaStream_t>(stream)>>>(m, a);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}
