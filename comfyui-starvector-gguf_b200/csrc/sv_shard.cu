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
// Wire formats (int32):
//   records (sv_pack_slice, one record per shard and row):
//     [0, C)      warped scores (float bits), the slice's kept tokens in index order
//     [C, 2C)     their global vocabulary indices
//     2C          kept count of the slice (may exceed C: the list was truncated)
//     2C + 1      the slice's status (SV_ST_*)
//   blocks (one per shard, written directly by the slice's sv_sample_step):
//     [0, RC)          warped scores (float bits) [rows][C]
//     [RC, 2RC)        slice-local indices [rows][C] (shard s adds s * slice_stride)
//     [2RC, 2RC + R)   kept counts
//     [2RC + R, 2RC + 2R) statuses
#include <cuda_runtime.h>

#include <cstdint>

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
  // Beam mode (ws != nullptr): the log_softmax stage's all-reduced statistics, and
  // the kept lists written to a beam workspace (header, ids, values) of ws_cap
  // entries a beam instead of a draw; out_score receives the kept log-probs.
  const float* gmax;
  const int32_t* gflags;
  unsigned char* ws;
  int ws_cap;
  float* out_score;
  // Blocked input (blocked != 0): shard s's block at packed + s * (2 rows cap +
  // 2 rows), its indices offset by s * slice_stride.
  int blocked, slice_stride;
};

struct __align__(16) MergeShared {
  BlockScratch<MNT> bs;
  int n, err, overflow;
  float wmx[MNT / 32];  // warps' largest candidates (the small finish's M)
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
    sh.err = 0;
    sh.overflow = 0;
  }
  __syncthreads();
  // Union of the shards' lists, in shard order.  A shard without a finite score
  // contributes nothing; any other shard error is the row's.  All shards' counts
  // and statuses are read at once, their offsets come from one scan, then every
  // thread copies candidates of any shard: three barriers whatever the shard count.
  int* take = sh.si;  // shard s's entries in the union (until leader_fast)
  int* base = sh.fi;  // and where they start
  auto shard_row = [&](int sd, const int32_t*& r, const int32_t*& ids, int& cnt, int& st, int& off) {
    if (m.blocked) {
      const int32_t* blk = m.packed + (int64_t)sd * (2 * (int64_t)m.rows * m.cap + 2 * m.rows);
      r = blk + (int64_t)row * m.cap;
      ids = blk + (int64_t)m.rows * m.cap + (int64_t)row * m.cap;
      cnt = blk[2 * (int64_t)m.rows * m.cap + row];
      st = blk[2 * (int64_t)m.rows * m.cap + m.rows + row];
      off = sd * m.slice_stride;
    } else {
      r = m.packed + ((int64_t)sd * m.rows + row) * rec;
      ids = r + m.cap;
      cnt = r[2 * m.cap];
      st = r[2 * m.cap + 1];
      off = 0;
    }
  };
  for (int sd = tid; sd < m.shards; sd += MNT) {
    const int32_t *r, *ids;
    int cnt, st, off;
    shard_row(sd, r, ids, cnt, st, off);
    int t = 0;
    if (st == ST_OK) {
      if (cnt > m.cap) atomicOr(&sh.overflow, 1);
      t = cnt < m.cap ? cnt : m.cap;
    } else if (st != ST_ALLNEGINF) {
      atomicOr(&sh.err, 1 << st);
    }
    take[sd] = t;
  }
  __syncthreads();
  if (tid < 32) {  // exclusive scan of the takes, 32 shards per pass
    int carry = 0;
    for (int s0 = 0; s0 < m.shards; s0 += 32) {
      const int sd = s0 + tid;
      const int t = sd < m.shards ? take[sd] : 0;
      int incl = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      if (sd < m.shards) base[sd] = carry + incl - t;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (tid == 0) sh.n = carry;
  }
  __syncthreads();
  for (int j = tid; j < m.shards * m.cap; j += MNT) {
    const int sd = j / m.cap, k = j - sd * m.cap;
    if (k >= take[sd]) continue;
    const int32_t *r, *ids;
    int cnt, st, off;
    shard_row(sd, r, ids, cnt, st, off);
    sh.cv[base[sd] + k] = __int_as_float(r[k]);
    sh.ci[base[sd] + k] = ids[k] + off;
  }
  __syncthreads();
  const int n = sh.n;
  int status = sh.err ? first_err(sh.err) : (sh.overflow ? ST_SHARD_OVERFLOW : (n == 0 ? ST_ALLNEGINF : ST_OK));
  if (m.ws) {
    // The log_softmax stage's status comes first (a NaN, else +inf, else no finite
    // logit in the whole row): the slices' steps ran on its meaningless output.
    const int fl = m.gflags[row];
    const float M = m.gmax[row];
    if (fl >= 2) status = ST_NAN;
    else if (fl == 1) status = ST_POSINF;
    else if (M == Elem<float>::neg_inf()) status = ST_ALLNEGINF;
  }
  Kept kept = {0, 0.0f, 0};
  int64_t token = -1;
  if (status == ST_OK) {
    const int mm = prefilter<MNT>(sh.bs, sh.cv, sh.ci, n, a.kk, sh.fv, sh.fi);
    if (!m.ws && mm <= 64) {
      // Few candidates: the batched kernel's finish, two threads per candidate
      // (its scratch over the sorted-list region, unused on this path).
      static_assert(sizeof(SmallFin) <= sizeof(float) * kMergeMax, "the small finish's state lies over sv");
      float mx = tid < mm ? sh.fv[tid] : Elem<float>::neg_inf();
      mx = warp_max_nan(mx);
      if ((tid & 31) == 0) sh.wmx[tid >> 5] = mx;
      __syncthreads();
      const float M = fmaxf(sh.wmx[0], sh.wmx[1]);
      int64_t tok = -1;
      const Kept kp = finish_small<MNT>(a, sh.fv, sh.fi, mm, M, m.uniforms[row], &tok, sh.fi, sh.fv,
                                        *reinterpret_cast<SmallFin*>(sh.sv));
      const float Sf = fix_to_float(kp.tot);
      for (int j = tid; j < kp.n && j < m.out_cap; j += MNT) {
        if (m.out_idx) m.out_idx[(int64_t)row * m.out_cap + j] = sh.fi[j];
        if (m.out_prob) m.out_prob[(int64_t)row * m.out_cap + j] = __fdiv_rn(sv_exp(__fsub_rn(sh.fv[j], kp.M)), Sf);
      }
      if (tid == 0) {
        m.out_token[row] = tok;
        if (m.out_count) m.out_count[row] = kp.n;
        if (m.out_status) m.out_status[row] = ST_OK;
      }
      return;
    }
    int* kidx = sh.ci;
    float* kval = sh.cv;
    kept = leader_fast<MNT>(a, sh.bs, sh.fv, sh.fi, mm, sh.sv, sh.si, reinterpret_cast<uint64_t*>(sh.fv),
                            reinterpret_cast<uint64_t*>(sh.cv), kidx, kval);
    if (m.ws) {
      int* wi = reinterpret_cast<int*>(m.ws + sizeof(BeamWsHeader)) + (int64_t)row * m.ws_cap;
      float* wv = reinterpret_cast<float*>(m.ws + sizeof(BeamWsHeader) + (size_t)m.rows * m.ws_cap * 4) +
                  (int64_t)row * m.ws_cap;
      for (int j = tid; j < kept.n; j += MNT) {
        wi[j] = kidx[j];
        wv[j] = kval[j];
        if (j < m.out_cap) {
          if (m.out_idx) m.out_idx[(int64_t)row * m.out_cap + j] = kidx[j];
          if (m.out_score) m.out_score[(int64_t)row * m.out_cap + j] = kval[j];
        }
      }
    }
  }
  if (m.ws) {
    if (tid == 0) {
      BeamWsHeader* hdr = reinterpret_cast<BeamWsHeader*>(m.ws);
      hdr->status[row] = status;
      hdr->count[row] = kept.n;
      if (m.out_count) m.out_count[row] = kept.n;
    }
    return;
  }
  if (status == ST_OK) {
    int* kidx = sh.ci;
    float* kval = sh.cv;
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

// Vocab-sharded beam step, one rank's slice (one block per beam): the maximum and
// NaN / +inf flags (global_max == nullptr), else the exact fixed-point sum of
// exp(x - M) for the all-reduced maximum M (the same arithmetic as the row
// kernel's log_softmax, runtime_shared.py:230).
template <typename TIn>
__global__ void __launch_bounds__(MNT) slice_stats_kernel(const TIn* x, int64_t stride, int len, const float* gmax,
                                                          float* out_max, int32_t* out_flags,
                                                          unsigned long long* out_sum) {
  __shared__ BlockScratch<MNT> bs;
  const int row = blockIdx.x, tid = threadIdx.x;
  const TIn* p = x + row * stride;
  const float PINF = __int_as_float(0x7f800000);
  if (!gmax) {
    float mx = Elem<float>::neg_inf();
    int nan = 0, inf = 0;
    for (int i = tid; i < len; i += MNT) {
      const float v = Elem<TIn>::to_f(p[i]);
      mx = max_nan(mx, v);
      nan |= v != v;
      inf |= v == PINF;
    }
    mx = block_max_nan<MNT>(bs, mx);
    nan = __syncthreads_or(nan);
    inf = __syncthreads_or(inf);
    if (tid == 0) {
      out_max[row] = mx;
      out_flags[row] = nan ? 2 : (inf ? 1 : 0);
    }
    return;
  }
  const float M = gmax[row];
  const bool ok = M == M && M != PINF && M != Elem<float>::neg_inf();
  uint64_t sum = 0;
  if (ok)
    for (int i = tid; i < len; i += MNT) sum += fixw(sv_exp(__fsub_rn(Elem<TIn>::to_f(p[i]), M)));
  sum = block_sum_u64<MNT>(bs, sum);
  if (tid == 0) out_sum[row] = sum;
}

// The slice's log-probabilities (x - M) - ln(S 2^-44) (runtime_shared.py:230), as
// the row kernel forms them.  Grid (blocks per beam, beams).
template <typename TIn>
__global__ void __launch_bounds__(MNT) slice_logprob_kernel(const TIn* x, int64_t stride, int len, const float* gmax,
                                                            const unsigned long long* gsum, float* out,
                                                            int64_t ostride) {
  __shared__ float sL;
  const int row = blockIdx.y;
  if (threadIdx.x == 0) sL = gsum[row] ? log_fixed(gsum[row]) : 0.0f;
  __syncthreads();
  const float M = gmax[row], Lg = sL;
  const TIn* p = x + row * stride;
  float* o = out + row * ostride;
  for (int i = blockIdx.x * MNT + threadIdx.x; i < len; i += gridDim.x * MNT)
    o[i] = __fsub_rn(__fsub_rn(Elem<TIn>::to_f(p[i]), M), Lg);
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

namespace {

int merge_sample(const int32_t* packed, int blocked, int32_t slice_stride, int32_t shards, int32_t rows,
                 int32_t capacity, const float* uniforms, double top_p, int32_t top_k, int32_t keep,
                 int64_t* out_token, int32_t* out_count, int32_t* out_idx, float* out_prob, int32_t out_capacity,
                 int32_t* out_status, void* stream) {
  if (!packed || !uniforms || !out_token) return SV_E_ARG;
  if (out_capacity > 0 && !out_idx && !out_prob) return SV_E_ARG;
  if (shards < 1 || rows < 1 || capacity < 1 || (int64_t)shards * capacity > kMergeMax || out_capacity < 0)
    return SV_E_SHAPE;
  if (blocked && (slice_stride < 1 || (int64_t)(shards - 1) * slice_stride > INT32_MAX)) return SV_E_SHAPE;
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
  m.blocked = blocked;
  m.slice_stride = slice_stride;
  merge_kernel<<<rows, MNT, 0, static_cast<cudaStream_t>(stream)>>>(m, a);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}

}  // namespace

// Merges the all-gathered per-shard kept lists of a vocab-sharded sample step; see
// include/starvector_sampling.h.
extern "C" int sv_merge_shards(const int32_t* packed, int32_t shards, int32_t rows, int32_t capacity,
                               const float* uniforms, double top_p, int32_t top_k, int32_t keep,
                               int64_t* out_token, int32_t* out_count, int32_t* out_idx, float* out_prob,
                               int32_t out_capacity, int32_t* out_status, void* stream) {
  return merge_sample(packed, 0, 0, shards, rows, capacity, uniforms, top_p, top_k, keep, out_token, out_count,
                      out_idx, out_prob, out_capacity, out_status, stream);
}

// The same merge over the all-gathered slice blocks; see include/starvector_sampling.h.
extern "C" int sv_merge_slices(const int32_t* blocks, int32_t shards, int32_t rows, int32_t capacity,
                               int32_t slice_stride, const float* uniforms, double top_p, int32_t top_k,
                               int32_t keep, int64_t* out_token, int32_t* out_count, int32_t* out_idx,
                               float* out_prob, int32_t out_capacity, int32_t* out_status, void* stream) {
  return merge_sample(blocks, 1, slice_stride, shards, rows, capacity, uniforms, top_p, top_k, keep, out_token,
                      out_count, out_idx, out_prob, out_capacity, out_status, stream);
}

// ------------------------------------------------- vocab-sharded beam step (C ABI)

namespace {

template <typename TIn>
cudaError_t launch_slice_stats(const void* x, int64_t stride, int beams, int len, const float* gmax, float* out_max,
                               int32_t* out_flags, unsigned long long* out_sum, cudaStream_t stream) {
  slice_stats_kernel<TIn><<<beams, MNT, 0, stream>>>(static_cast<const TIn*>(x), stride, len, gmax, out_max,
                                                      out_flags, out_sum);
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_slice_logprobs(const void* x, int64_t stride, int beams, int len, const float* gmax,
                                  const unsigned long long* gsum, float* out, int64_t ostride, cudaStream_t stream) {
  const int per_beam = (len + 4 * MNT - 1) / (4 * MNT);
  slice_logprob_kernel<TIn><<<dim3(per_beam, beams), MNT, 0, stream>>>(static_cast<const TIn*>(x), stride, len, gmax,
                                                                        gsum, out, ostride);
  return cudaGetLastError();
}

}  // namespace

// Statistics of one rank's vocabulary slice for the sharded beam step; see
// include/starvector_sampling.h.
extern "C" int sv_beam_slice_stats(const void* logits, int32_t logits_dtype, int32_t beams, int32_t slice_len,
                                   int64_t logits_row_stride, const float* global_max, float* out_max,
                                   int32_t* out_flags, uint64_t* out_sum, void* stream) {
  if (!logits) return SV_E_ARG;
  if (global_max ? !out_sum : (!out_max || !out_flags)) return SV_E_ARG;
  if (beams < 1 || beams > kMaxBeams || slice_len < 1 || logits_row_stride < 0) return SV_E_SHAPE;
  if (beams > 1 && logits_row_stride < slice_len) return SV_E_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* sum = reinterpret_cast<unsigned long long*>(out_sum);
  cudaError_t e;
  if (logits_dtype == DT_F32)
    e = launch_slice_stats<float>(logits, logits_row_stride, beams, slice_len, global_max, out_max, out_flags, sum, s);
  else if (logits_dtype == DT_F16)
    e = launch_slice_stats<__half>(logits, logits_row_stride, beams, slice_len, global_max, out_max, out_flags, sum, s);
  else if (logits_dtype == DT_BF16)
    e = launch_slice_stats<__nv_bfloat16>(logits, logits_row_stride, beams, slice_len, global_max, out_max, out_flags,
                                          sum, s);
  else
    return SV_E_DTYPE;
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

// The slice's log-probabilities from the all-reduced statistics; see
// include/starvector_sampling.h.
extern "C" int sv_beam_slice_logprobs(const void* logits, int32_t logits_dtype, int32_t beams, int32_t slice_len,
                                      int64_t logits_row_stride, const float* global_max, const uint64_t* global_sum,
                                      float* out, int64_t out_row_stride, void* stream) {
  if (!logits || !global_max || !global_sum || !out) return SV_E_ARG;
  if (beams < 1 || beams > kMaxBeams || slice_len < 1 || logits_row_stride < 0) return SV_E_SHAPE;
  if (beams > 1 && (logits_row_stride < slice_len || out_row_stride < slice_len)) return SV_E_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* gs = reinterpret_cast<const unsigned long long*>(global_sum);
  cudaError_t e;
  if (logits_dtype == DT_F32)
    e = launch_slice_logprobs<float>(logits, logits_row_stride, beams, slice_len, global_max, gs, out, out_row_stride, s);
  else if (logits_dtype == DT_F16)
    e = launch_slice_logprobs<__half>(logits, logits_row_stride, beams, slice_len, global_max, gs, out, out_row_stride,
                                      s);
  else if (logits_dtype == DT_BF16)
    e = launch_slice_logprobs<__nv_bfloat16>(logits, logits_row_stride, beams, slice_len, global_max, gs, out,
                                             out_row_stride, s);
  else
    return SV_E_DTYPE;
  return e == cudaSuccess ? SV_OK : SV_E_CUDA;
}

// Workspace of sv_merge_beam_shards: the beam workspace layout with
// shards * capacity kept entries a beam.
extern "C" size_t sv_merge_beam_shards_workspace_bytes(int32_t beams, int32_t shards, int32_t capacity) {
  if (beams < 1 || shards < 1 || capacity < 1) return 0;
  return sizeof(BeamWsHeader) + (size_t)beams * (size_t)shards * (size_t)capacity * 16;
}

namespace {

int merge_beam(const int32_t* packed, int blocked, int32_t slice_stride, int32_t shards, int32_t beams,
               int32_t capacity, int32_t vocab, const float* global_max, const int32_t* global_flags,
               const float* running_scores, const float* uniforms, int32_t num_picks, double top_p, int32_t top_k,
               int32_t keep, void* workspace, size_t workspace_bytes, int64_t* out_picks, float* out_pick_scores,
               int32_t* out_num_picks, int32_t* out_status, int32_t* out_kept_count, int32_t* out_kept_idx,
               float* out_kept_logprob, float* out_kept_prob, int32_t out_capacity, void* stream) {
  if (!packed || !global_max || !global_flags || !running_scores || !uniforms || !workspace || !out_picks ||
      !out_pick_scores || !out_num_picks || !out_status)
    return SV_E_ARG;
  if (out_capacity > 0 && !out_kept_idx && !out_kept_logprob && !out_kept_prob) return SV_E_ARG;
  if (shards < 1 || beams < 1 || beams > kMaxBeams || capacity < 1 || (int64_t)shards * capacity > kMergeMax ||
      vocab < 1 || out_capacity < 0)
    return SV_E_SHAPE;
  if (blocked && (slice_stride < 1 || (int64_t)(shards - 1) * slice_stride >= vocab)) return SV_E_SHAPE;
  if (num_picks < 1 || num_picks > 64) return SV_E_RANGE;
  if (!(top_p > 0.0 && top_p <= 1.0)) return SV_E_RANGE;
  if (top_k < 1 || top_k > kMaxTopK || keep < 1 || keep > kMaxTopK) return SV_E_RANGE;
  const int kk = top_k > keep ? top_k : keep;
  if (kk > capacity) return SV_E_RANGE;
  if (workspace_bytes < sv_merge_beam_shards_workspace_bytes(beams, shards, capacity)) return SV_E_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return SV_E_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RowArgs a = {};
  a.kk = kk;
  a.keep = keep;
  a.pthr = top_p < 1.0 ? (float)(1.0 - top_p) : 0.0f;
  MergeArgs m = {packed, shards, beams, capacity, uniforms, nullptr, out_kept_count, out_kept_idx, nullptr,
                 out_capacity, nullptr, global_max, global_flags, static_cast<unsigned char*>(workspace),
                 shards * capacity, out_kept_logprob};
  m.blocked = blocked;
  m.slice_stride = slice_stride;
  merge_kernel<<<beams, MNT, 0, s>>>(m, a);
  if (cudaGetLastError() != cudaSuccess) return SV_E_CUDA;
  RowArgs b = {};
  b.mode = MODE_BEAM;
  b.rows = beams;
  b.vocab = vocab;
  b.ws = static_cast<unsigned char*>(workspace);
  b.ws_cap = shards * capacity;
  b.running = running_scores;
  b.uniforms = uniforms;
  b.npick = num_picks;
  b.out_picks = out_picks;
  b.out_pick_scores = out_pick_scores;
  b.out_npicks = out_num_picks;
  b.out_status = out_status;
  b.out_prob = out_kept_prob;
  b.out_cap = out_capacity;
  return launch_beam_merge(b, s) == cudaSuccess ? SV_OK : SV_E_CUDA;
}

}  // namespace

// Merge side of the vocab-sharded beam step; see include/starvector_sampling.h.
extern "C" int sv_merge_beam_shards(const int32_t* packed, int32_t shards, int32_t beams, int32_t capacity,
                                    int32_t vocab, const float* global_max, const int32_t* global_flags,
                                    const float* running_scores, const float* uniforms, int32_t num_picks,
                                    double top_p, int32_t top_k, int32_t keep, void* workspace,
                                    size_t workspace_bytes, int64_t* out_picks, float* out_pick_scores,
                                    int32_t* out_num_picks, int32_t* out_status, int32_t* out_kept_count,
                                    int32_t* out_kept_idx, float* out_kept_logprob, float* out_kept_prob,
                                    int32_t out_capacity, void* stream) {
  return merge_beam(packed, 0, 0, shards, beams, capacity, vocab, global_max, global_flags, running_scores, uniforms,
                    num_picks, top_p, top_k, keep, workspace, workspace_bytes, out_picks, out_pick_scores,
                    out_num_picks, out_status, out_kept_count, out_kept_idx, out_kept_logprob, out_kept_prob,
                    out_capacity, stream);
}

// The same over the all-gathered slice blocks; see include/starvector_sampling.h.
extern "C" int sv_merge_beam_slices(const int32_t* blocks, int32_t shards, int32_t beams, int32_t capacity,
                                    int32_t slice_stride, int32_t vocab, const float* global_max,
                                    const int32_t* global_flags, const float* running_scores, const float* uniforms,
                                    int32_t num_picks, double top_p, int32_t top_k, int32_t keep, void* workspace,
                                    size_t workspace_bytes, int64_t* out_picks, float* out_pick_scores,
                                    int32_t* out_num_picks, int32_t* out_status, int32_t* out_kept_count,
                                    int32_t* out_kept_idx, float* out_kept_logprob, float* out_kept_prob,
                                    int32_t out_capacity, void* stream) {
  return merge_beam(blocks, 1, slice_stride, shards, beams, capacity, vocab, global_max, global_flags, running_scores,
                    uniforms, num_picks, top_p, top_k, keep, workspace, workspace_bytes, out_picks, out_pick_scores,
                    out_num_picks, out_status, out_kept_count, out_kept_idx, out_kept_logprob, out_kept_prob,
                    out_capacity, stream);
}
