// sv_block.cuh -- block-level building blocks shared by the row kernels:
// reductions and scans, the bulk-copy / mbarrier helpers, the lower bound of the
// k-th largest score, and the routines that finish a row from its candidates
// (top-k with ties, top-p, the draw) or from the whole row (the general path).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

template <int NT>
struct BlockScratch {
  unsigned long long bsum[NT / 32];
  float bmax[NT / 32];
  int bint[NT / 32];
  int iscr[NT / 32];
  int flag, flag2;
  unsigned long long u64a;
  float fval;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------- reductions

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int NT>
__device__ uint64_t block_sum_u64(BlockScratch<NT>& bs, uint64_t v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_u64(v);
  __syncthreads();
  if (lane == 0) bs.bsum[warp] = v;
  __syncthreads();
  uint64_t t = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += bs.bsum[w];
  return t;
}

template <int NT>
__device__ int block_sum_int(BlockScratch<NT>& bs, int v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_int(v);
  __syncthreads();
  if (lane == 0) bs.bint[warp] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += bs.bint[w];
  return t;
}

template <int NT>
__device__ float block_max_nan(BlockScratch<NT>& bs, float v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max_nan(v);
  __syncthreads();
  if (lane == 0) bs.bmax[warp] = v;
  __syncthreads();
  float t = bs.bmax[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) t = max_nan(t, bs.bmax[w]);
  return t;
}

// Exclusive block scan of one value per thread; *total receives the block sum.
template <int NT, typename T>
__device__ T block_excl_scan(T v, T* scratch /* NT/32 */, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  T before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    T s = scratch[w];
    if (w < warp) before += s;
    all += s;
  }
  *total = all;
  return before + incl - v;
}

// In-place inclusive scan of a[0, n) by the whole block (each thread a run).
template <int NT>
__device__ void block_scan_inplace_u64(BlockScratch<NT>& bs, uint64_t* a, int n) {
  const int per = (n + NT - 1) / NT;
  const int b = threadIdx.x * per;
  unsigned long long s = 0;
  for (int q = 0; q < per; ++q)
    if (b + q < n) {
      s += a[b + q];
      a[b + q] = s;
    }
  unsigned long long tot;
  const unsigned long long ex = block_excl_scan<NT, unsigned long long>(s, bs.bsum, &tot);
  for (int q = 0; q < per; ++q)
    if (b + q < n) a[b + q] += ex;
  __syncthreads();
}

// ------------------------------------------------------ bulk copy + mbarrier

__device__ __forceinline__ void mbar_init(void* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(void* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(void* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Orders earlier generic-proxy shared-memory accesses (the block's, after a block
// barrier) before later async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk copy global -> this CTA's shared memory, completing on `bar`.  dst, src and
// bytes must be multiples of 16 (the callers' layouts guarantee it).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, void* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// One try_wait; the thread may be suspended up to ~1 ms (it resumes as soon as the
// phase completes), so a waiting warp issues few instructions.
__device__ __forceinline__ bool mbar_try(uint32_t b, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(b), "r"(phase), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase: gives up after limit_ns of global time, ~1 s
// by default (the timer is read only once the phase is found incomplete).
__device__ inline bool mbar_wait(void* bar, uint32_t phase, uint64_t limit_ns = 1000000000ull) {
  const uint32_t b = smem_u32(bar);
  if (mbar_try(b, phase)) return true;
  const uint64_t t0 = gtimer_ns();
  for (;;) {
    if (mbar_try(b, phase)) return true;
    if (gtimer_ns() - t0 > limit_ns) return false;
  }
}

// ------------------------------------------------------------------ units
// A unit is 16 bytes of staged logits: 4 fp32 or 8 fp16/bf16 values.

template <typename TIn> struct UnitIO;
template <> struct UnitIO<float> {
  static constexpr int E = 4;
  __device__ static void load(const float* d, int u, float (&v)[E]) {
    float4 t = reinterpret_cast<const float4*>(d)[u];
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  }
  __device__ static void store(float* d, int u, const float (&v)[E]) {
    reinterpret_cast<float4*>(d)[u] = make_float4(v[0], v[1], v[2], v[3]);
  }
  __device__ static uint32_t mask(const unsigned char* m, int u) { return reinterpret_cast<const uint32_t*>(m)[u]; }
};
template <typename H> struct UnitIOHalf {
  static constexpr int E = 8;
  __device__ static void load(const H* d, int u, float (&v)[E]) {
    uint4 t = reinterpret_cast<const uint4*>(d)[u];
    const H* h = reinterpret_cast<const H*>(&t);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = Elem<H>::to_f(h[e]);
  }
  __device__ static void store(H*, int, const float (&)[E]) {}
  __device__ static uint64_t mask(const unsigned char* m, int u) { return reinterpret_cast<const uint64_t*>(m)[u]; }
};
template <> struct UnitIO<__half> : UnitIOHalf<__half> {};
template <> struct UnitIO<__nv_bfloat16> : UnitIOHalf<__nv_bfloat16> {};

__device__ __forceinline__ bool mask_bit(uint64_t m, int e) { return (m >> (8 * e)) & 0xffu; }

// ---------------------------------------------------------------- history

__device__ __forceinline__ int64_t hist_id(const RowArgs& a, int64_t row, int64_t j) {
  if (a.hist_kind == HIST_IDS32) return reinterpret_cast<const int32_t*>(a.hist)[row * a.hist_stride + j];
  return reinterpret_cast<const int64_t*>(a.hist)[row * a.hist_stride + j];
}

// Valid history prefix of a row: history_len[row] clamped to [0, history_cols].
__device__ __forceinline__ int64_t hist_length(const RowArgs& a, int64_t row) {
  int64_t L = a.hist_len ? (int64_t)a.hist_len[row] : (int64_t)a.hist_cols;
  if (L > a.hist_cols) L = a.hist_cols;
  return L < 0 ? 0 : L;
}

__device__ __forceinline__ bool seen_global(const RowArgs& a, int64_t row, int64_t i) {
  if (a.hist_kind == HIST_MASK8) return reinterpret_cast<const unsigned char*>(a.hist)[row * a.hist_stride + i] != 0;
  if (a.hist_kind == HIST_BITS32)
    return (reinterpret_cast<const uint32_t*>(a.hist)[row * a.hist_stride + (i >> 5)] >> (i & 31)) & 1u;
  return false;
}

// Sets m[id - lo] for the ids in [lo, hi) among h[0, L) (h in global or shared
// memory: plain loads).  Loads are issued in batches of 8 per thread before any
// store so their latencies overlap.  Returns the ST_HISTORY error bit for ids
// outside [0, V).
template <int NT, typename Id>
__device__ __forceinline__ int mark_ids(const Id* h, int64_t L, int64_t V, int64_t lo, int64_t hi,
                                        unsigned char* m) {
  constexpr int U = 8;
  int err = 0;
  for (int64_t base = 0; base < L; base += (int64_t)NT * U) {
    int64_t id[U];
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const int64_t j = base + threadIdx.x + (int64_t)q * NT;
      id[q] = j < L ? (int64_t)h[j] : lo - 1;
    }
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const int64_t j = base + threadIdx.x + (int64_t)q * NT;
      if (j < L && (id[q] < 0 || id[q] >= V)) err |= 1 << ST_HISTORY;
      else if (id[q] >= lo && id[q] < hi) m[id[q] - lo] = 1;
    }
  }
  return err;
}

// ------------------------------------------------------------ lower bound tau

// tau lowered by |tau| 2^-16 + T 2^-140 + 2^-140 (towards -inf).  An element whose
// tempered score can equal the k-th largest tempered score lies within T * ulp of
// the k-th largest penalised score, far inside this margin.
__device__ __forceinline__ float lower_tau(float tau, float T) {
  if (tau == Elem<float>::neg_inf()) return tau;
  float m = __fadd_ru(__fmul_ru(fabsf(tau), 1.52587890625e-05f), __fmul_ru(T, 7.174648137343064e-43f));
  m = __fadd_ru(m, 7.174648137343064e-43f);
  return __fsub_rd(tau, m);
}

// The kk-th largest of g[0, G) (G <= NT, kk <= G) by rank counting, one value per
// thread; NaN / +inf among g set error bits in *err.  Returns the lowered bound
// (all threads).  With G disjoint groups, kk of them have a maximum >= this value,
// so it is a lower bound of the kk-th largest element.
template <int NT>
__device__ float tau_from_groups(BlockScratch<NT>& bs, const float* g, int G, int kk, float T, int* err) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    bs.flag = 0;
    bs.fval = Elem<float>::neg_inf();
  }
  __syncthreads();
  if (tid < G) {
    const float v = g[tid];
    if (v != v) atomicOr(&bs.flag, 1 << ST_NAN);
    else if (v == __int_as_float(0x7f800000)) atomicOr(&bs.flag, 1 << ST_POSINF);
    const uint32_t kt = ord_key(v);
    int gt = 0, ge = 0;
    for (int j = 0; j < G; ++j) {
      const uint32_t kj = ord_key(g[j]);
      gt += kj > kt;
      ge += kj >= kt;
    }
    if (gt < kk && kk <= ge) bs.fval = v;
  }
  __syncthreads();
  const int e = bs.flag;
  const float tau = bs.fval;
  if (tid == 0 && e) atomicOr(err, e);
  __syncthreads();
  return lower_tau(tau, T);
}

__device__ __forceinline__ int first_err(int e) {
  for (int s = 1; s < 8; ++s)
    if (e & (1 << s)) return s;
  return ST_OK;
}

// ------------------------------------------------------------- finish: fast

struct Kept {
  int n;         // kept count
  float M;       // maximum of the warped scores
  uint64_t tot;  // fixed-point mass of the kept entries
};

// Exact kk-th largest of n candidate scores by counting, then compaction of the
// candidates >= it into (sv, si).  Returns their count m (>= kk unless fewer than
// kk candidates exist, when all are kept).
template <int NT>
__device__ int prefilter(BlockScratch<NT>& bs, const float* cv, const int* ci, int n, int kk, float* sv, int* si) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    bs.fval = Elem<float>::neg_inf();
    bs.flag = 0;
  }
  __syncthreads();
  if (n >= kk) {
    for (int t = tid; t < n; t += NT) {
      const float v = cv[t];
      int gt = 0, ge = 0;
      for (int j = 0; j < n; ++j) {
        const float w = cv[j];
        gt += w > v;
        ge += w >= v;
      }
      if (gt < kk && kk <= ge) bs.fval = v;
    }
  }
  __syncthreads();
  const float thr = bs.fval;
  for (int t = tid; t < n; t += NT) {
    const float v = cv[t];
    if (v >= thr) {
      const int s = atomicAdd(&bs.flag, 1);
      sv[s] = v;
      si[s] = ci[t];
    }
  }
  __syncthreads();
  const int m = bs.flag;
  __syncthreads();
  return m;
}

// Top-k threshold with ties, top-p and the index-ordered kept list from n
// candidates (in_val, in_idx), which must contain every entry >= the k-th largest.
//   sval, sidx: n floats / ints; W: n u64 (may alias in_val/in_idx); P: n u64 (must
//   not alias in_val/in_idx).  kidx, kval: the kept list (may alias P).
template <int NT>
__device__ Kept leader_fast(const RowArgs& a, BlockScratch<NT>& bs, const float* in_val, const int* in_idx, int n,
                            float* sval, int* sidx, uint64_t* W, uint64_t* P, int* kidx, float* kval) {
  const int tid = threadIdx.x;
  // (a) ascending order by (value, index): rank counting over 64-bit ordered keys
  //     (distinct, since indices are), staged in P.
  for (int t = tid; t < n; t += NT) P[t] = ((uint64_t)ord_key(in_val[t]) << 32) | (uint32_t)in_idx[t];
  __syncthreads();
  for (int t = tid; t < n; t += NT) {
    const uint64_t kt = P[t];
    int rank = 0, j = 0;
    for (; j + 4 <= n; j += 4) rank += (P[j] < kt) + (P[j + 1] < kt) + (P[j + 2] < kt) + (P[j + 3] < kt);
    for (; j < n; ++j) rank += P[j] < kt;
    sval[rank] = in_val[t];
    sidx[rank] = in_idx[t];
  }
  __syncthreads();
  // (b) exact k-th largest with ties: survivors are sorted positions [f0, n).
  const int kk = a.kk;
  const float thr = n >= kk ? sval[n - kk] : Elem<float>::neg_inf();
  if (tid == 0) bs.flag = 0;
  __syncthreads();
  for (int j = tid; j < n; j += NT)
    if (sval[j] >= thr && (j == 0 || sval[j - 1] < thr)) bs.flag = j;
  __syncthreads();
  const int f0 = bs.flag;
  const int m = n - f0;
  const float M = sval[n - 1];
  // (c) weights
  for (int j = f0 + tid; j < n; j += NT) W[j] = fixw(sv_exp(__fsub_rn(sval[j], M)));
  __syncthreads();
  uint64_t lsum = 0;
  for (int j = f0 + tid; j < n; j += NT) lsum += W[j];
  const uint64_t total = block_sum_u64<NT>(bs, lsum);
  // (d) top-p: remove the ascending prefix whose mass is <= floor(total * pthr),
  //     never the last `keep` (runtime_shared.py:184-185).
  int r = 0;
  uint64_t removed = 0;
  if (a.pthr > 0.0f) {
    for (int j = tid; j < m; j += NT) P[j] = W[f0 + j];
    __syncthreads();
    block_scan_inplace_u64<NT>(bs, P, m);
    const uint64_t thrW = mulfloor(total, a.pthr);
    if (tid == 0) bs.flag = m;
    __syncthreads();
    for (int j = tid; j < m; j += NT)
      if (P[j] > thrW && (j == 0 || P[j - 1] <= thrW)) bs.flag = j;
    __syncthreads();
    r = bs.flag;
    const int cap = m - a.keep > 0 ? m - a.keep : 0;
    if (r > cap) r = cap;
    removed = r > 0 ? P[r - 1] : 0;
    __syncthreads();
  }
  const int k0 = f0 + r;
  const int mk = n - k0;
  // (e) kept entries in index order.
  for (int t = k0 + tid; t < n; t += NT) {
    const int it = sidx[t];
    int rank = 0;
    for (int j = k0; j < n; ++j) rank += sidx[j] < it;
    kidx[rank] = it;
    kval[rank] = sval[t];
  }
  __syncthreads();
  Kept k;
  k.n = mk;
  k.M = M;
  k.tot = total - removed;
  return k;
}

// The sample-mode draw over the index-ordered kept list: the first kept index whose
// inclusive prefix of fixed-point weights exceeds floor(u * total).  Wk: n u64.
template <int NT>
__device__ int64_t draw_kept(BlockScratch<NT>& bs, const int* kidx, const float* kval, const Kept& k, float u,
                             uint64_t* Wk) {
  const int tid = threadIdx.x;
  for (int j = tid; j < k.n; j += NT) Wk[j] = fixw(sv_exp(__fsub_rn(kval[j], k.M)));
  __syncthreads();
  block_scan_inplace_u64<NT>(bs, Wk, k.n);
  const uint64_t Tu = mulfloor(k.tot, u);
  if (tid == 0) bs.flag = k.n - 1;
  __syncthreads();
  for (int j = tid; j < k.n; j += NT)
    if (Wk[j] > Tu && (j == 0 || Wk[j - 1] <= Tu)) bs.flag = j;
  __syncthreads();
  const int64_t token = kidx[bs.flag];
  __syncthreads();
  return token;
}

// ------------------------------------------------------ finish: one warp
// The same finish as leader_fast + draw_kept for at most 32 * N candidates, done
// by the calling warp alone in registers (no block barriers).  Lane l holds the
// positions s * 32 + l, s < N.

// Ascending bitonic sort of 32 * N keys in one warp.
template <int N>
__device__ __forceinline__ void warp_sort(uint64_t (&x)[N]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32 * N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {  // partners in the same lane: registers s and s | (j / 32)
#pragma unroll
        for (int s = 0; s < N; ++s) {
          if ((s & (j >> 5)) == 0) {
            const int t = s | (j >> 5);
            const bool asc = ((s * 32) & k) == 0;
            const uint64_t lo = x[s] < x[t] ? x[s] : x[t], hi = x[s] < x[t] ? x[t] : x[s];
            x[s] = asc ? lo : hi;
            x[t] = asc ? hi : lo;
          }
        }
      } else {
        const bool upper = (lane & j) != 0;
#pragma unroll
        for (int s = 0; s < N; ++s) {
          const uint64_t p = __shfl_xor_sync(0xffffffffu, x[s], j);
          // The lower position of an ascending pair (or the upper of a descending
          // one) keeps the minimum.
          const bool keep_min = (((s * 32 + lane) & k) == 0) != upper;
          x[s] = keep_min ? (x[s] < p ? x[s] : p) : (x[s] < p ? p : x[s]);
        }
      }
    }
  }
}

__device__ __forceinline__ uint64_t warp_incl_scan_u64(uint64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// The value at position p (per lane) of a per-position register set.  Every lane
// must call it.
template <int N, typename T>
__device__ __forceinline__ T warp_at(const T (&x)[N], int p) {
  T r = x[0];
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const T t = __shfl_sync(0xffffffffu, x[s], p & 31);
    if ((p >> 5) == s) r = t;
  }
  return r;
}

// First position (s * 32 + lane order) whose predicate holds, or `none`.
template <int N>
__device__ __forceinline__ int warp_first(const bool (&pr)[N], int none) {
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const unsigned b = __ballot_sync(0xffffffffu, pr[s]);
    if (b) return s * 32 + __ffs(b) - 1;
  }
  return none;
}

// Top-k threshold with ties (runtime_shared.py:180-181), top-p (:182-186) and the
// draw for m <= 32 * N candidates (fv: tempered scores, fi: indices; m >= 1), by
// the calling warp.  Returns the Kept summary (every lane), sets *token (every
// lane) and writes the kept list in index order to kidx / kval.
template <int N>
__device__ Kept warp_finish(const RowArgs& a, const float* fv, const int* fi, int m, float u, int64_t* token,
                            int* kidx, float* kval) {
  constexpr int C = 32 * N;
  const int lane = threadIdx.x & 31;
  const float NEG = Elem<float>::neg_inf();
  // (a) ascending (value, index) order; padding keys (0) sort first.
  uint64_t x[N];
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const int p = s * 32 + lane;
    x[s] = p < m ? ((uint64_t)ord_key(fv[p]) << 32) | (uint32_t)fi[p] : 0ull;
  }
  warp_sort<N>(x);
  float v[N];
#pragma unroll
  for (int s = 0; s < N; ++s) v[s] = key_to_float((uint32_t)(x[s] >> 32));
  // (b) k-th largest with ties: kept positions [f0, C).
  const float thr = m >= a.kk ? warp_at<N>(v, C - a.kk) : NEG;
  bool in[N];
#pragma unroll
  for (int s = 0; s < N; ++s) in[s] = s * 32 + lane >= C - m && v[s] >= thr;
  const int f0 = warp_first<N>(in, C - 1);
  const float M = __shfl_sync(0xffffffffu, v[N - 1], 31);
  // (c) weights and their ascending prefix sums.
  uint64_t w[N], P[N], carry = 0;
#pragma unroll
  for (int s = 0; s < N; ++s) {
    w[s] = in[s] ? fixw(sv_exp(__fsub_rn(v[s], M))) : 0ull;
    P[s] = carry + warp_incl_scan_u64(w[s]);
    carry = __shfl_sync(0xffffffffu, P[s], 31);
  }
  const uint64_t total = carry;
  // (d) top-p: the ascending prefix with mass <= floor(total * pthr) goes, never
  //     the last `keep`.
  int k0 = f0;
  uint64_t removed = 0;
  if (a.pthr > 0.0f) {
    const uint64_t thrW = mulfloor(total, a.pthr);
    bool c[N];
#pragma unroll
    for (int s = 0; s < N; ++s) c[s] = in[s] && P[s] > thrW;
    int r = warp_first<N>(c, C) - f0;
    const int cap = (C - f0) - a.keep > 0 ? (C - f0) - a.keep : 0;
    if (r > cap) r = cap;
    k0 = f0 + r;
    if (r > 0) removed = warp_at<N>(P, k0 - 1);
  }
  Kept kp;
  kp.n = C - k0;
  kp.M = M;
  kp.tot = total - removed;
  // (e) the kept entries in index order, then the draw over them.
  uint64_t y[N];
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const int p = s * 32 + lane;
    y[s] = p >= k0 ? ((uint64_t)(uint32_t)x[s] << 8) | (uint32_t)p : ~0ull;
  }
  warp_sort<N>(y);
  uint64_t Q[N];
  bool hit[N];
  const uint64_t Tu = mulfloor(kp.tot, u);
  carry = 0;
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const int q = s * 32 + lane;
    const int o = (int)(y[s] & 0xffu) & (C - 1);
    const uint64_t wq = warp_at<N>(w, o);  // every lane shuffles
    const float vq = warp_at<N>(v, o);
    Q[s] = carry + warp_incl_scan_u64(q < kp.n ? wq : 0ull);
    carry = __shfl_sync(0xffffffffu, Q[s], 31);
    hit[s] = q < kp.n && Q[s] > Tu;
    if (q < kp.n) {
      kidx[q] = (int)(y[s] >> 8);
      kval[q] = vq;
    }
  }
  const int qd = warp_first<N>(hit, kp.n - 1);
  *token = (int64_t)(warp_at<N>(y, qd) >> 8);
  __syncwarp();
  return kp;
}

// --------------------------------------------------------- finish: general
// The general path over the whole row from global memory (huge tie groups): an
// exact radix select of the k-th largest key, the tie group handled
// arithmetically (top-p removes its members lowest index first), and one
// index-ordered pass that emits the kept entries, draws the token (sample mode)
// and writes the dense output.
//   seen(i): the penalty applies to index i.  emit(pos, idx, value, Sf, M).
//   scratch: >= 4 KB of shared memory.
template <int NT, typename TIn, int MODE, typename SeenFn, typename Emit>
__device__ Kept leader_slow(const RowArgs& a, BlockScratch<NT>& bs, unsigned char* scratch, int64_t row, float bM,
                            float bL, float u, int64_t* token, SeenFn seen, Emit emit) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t V = a.vocab;
  const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
  uint32_t* hist = reinterpret_cast<uint32_t*>(scratch);  // 256 bins
  float* gval = reinterpret_cast<float*>(scratch + 1024);  // <= kMaxTopK
  int* gidx = reinterpret_cast<int*>(scratch + 1024 + 4 * kMaxTopK);
  float* gsv = reinterpret_cast<float*>(scratch + 1024 + 8 * kMaxTopK);
  int* gsi = reinterpret_cast<int*>(scratch + 1024 + 12 * kMaxTopK);
  const float rp = a.rep_penalty, T = a.temperature;
  auto F = [&](int64_t i) -> float {
    float x = Elem<TIn>::load(rowp + i);
    if (MODE == MODE_BEAM) x = __fsub_rn(__fsub_rn(x, bM), bL);
    if (seen(i)) x = penalize(x, rp);
    return temper(x, T);
  };
  const float NEG = Elem<float>::neg_inf();
  const int kk = a.kk;

  // Exact k-th largest key K by 8-bit radix select over the finite values.
  int nfin = 0;
  for (int64_t i = tid; i < V; i += NT) nfin += F(i) > NEG;
  nfin = block_sum_int<NT>(bs, nfin);
  uint32_t prefix = 0, pmask = 0;
  int need = kk;
  const bool have_thr = nfin >= kk;
  if (have_thr) {
    for (int round = 0; round < 4; ++round) {
      const int shf = 24 - 8 * round;
      for (int b = tid; b < 256; b += NT) hist[b] = 0;
      __syncthreads();
      for (int64_t i = tid; i < V; i += NT) {
        const float f = F(i);
        if (f > NEG) {
          const uint32_t k = ord_key(f);
          if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shf) & 255u], 1u);
        }
      }
      __syncthreads();
      if (warp == 0) {
        uint32_t c[8], s = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c[q] = hist[lane * 8 + q];
          s += c[q];
        }
        uint32_t incl = s;  // sum over lanes >= lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
          if (lane + o < 32) incl += t;
        }
        if (incl >= (uint32_t)need && incl - s < (uint32_t)need) {
          uint32_t above = incl - s;
          for (int q = 7; q >= 0; --q) {
            if (above + c[q] >= (uint32_t)need) {
              bs.flag = lane * 8 + q;
              bs.flag2 = (int)above;
              break;
            }
            above += c[q];
          }
        }
      }
      __syncthreads();
      prefix |= (uint32_t)bs.flag << shf;
      pmask |= 255u << shf;
      need -= bs.flag2;
      __syncthreads();
    }
  }
  const uint32_t K = prefix;
  const float thr = have_thr ? key_to_float(K) : NEG;

  // The tie group (key == K) is counted; the entries above it (< kk) collected.
  if (tid == 0) bs.flag = 0;
  __syncthreads();
  int neq = 0;
  for (int64_t i = tid; i < V; i += NT) {
    const float f = F(i);
    if (!(f > NEG)) continue;
    const uint32_t k = ord_key(f);
    if (have_thr && k == K) ++neq;
    else if (!have_thr || k > K) {
      const int s = atomicAdd(&bs.flag, 1);
      if (s < kMaxTopK) {
        gval[s] = f;
        gidx[s] = (int)i;
      }
    }
  }
  neq = block_sum_int<NT>(bs, neq);
  const int ngt = min(bs.flag, kMaxTopK);
  __syncthreads();
  for (int t = tid; t < ngt; t += NT) {
    const uint64_t kt = ((uint64_t)ord_key(gval[t]) << 32) | (uint32_t)gidx[t];
    int rank = 0;
    for (int j = 0; j < ngt; ++j) rank += (((uint64_t)ord_key(gval[j]) << 32) | (uint32_t)gidx[j]) < kt;
    gsv[rank] = gval[t];
    gsi[rank] = gidx[t];
  }
  __syncthreads();
  const float M = ngt > 0 ? gsv[ngt - 1] : thr;
  const uint64_t Wt = neq > 0 ? fixw(sv_exp(__fsub_rn(thr, M))) : 0;
  if (tid == 0) {
    uint64_t total = (uint64_t)neq * Wt;
    for (int g = 0; g < ngt; ++g) total += fixw(sv_exp(__fsub_rn(gsv[g], M)));
    const int m = neq + ngt;
    int r = 0;
    if (a.pthr > 0.0f) {
      const uint64_t thrW = mulfloor(total, a.pthr);
      const uint64_t req = Wt == 0 ? (uint64_t)neq : thrW / Wt;
      r = req < (uint64_t)neq ? (int)req : neq;
      if (r == neq) {
        uint64_t P = (uint64_t)neq * Wt;
        for (int g = 0; g < ngt; ++g) {
          P += fixw(sv_exp(__fsub_rn(gsv[g], M)));
          if (P <= thrW) ++r;
          else break;
        }
      }
      const int cap = m - a.keep > 0 ? m - a.keep : 0;
      if (r > cap) r = cap;
    }
    const int req2 = r < neq ? r : neq;
    const int rgt = r - req2;
    uint64_t kept = (uint64_t)(neq - req2) * Wt;
    for (int g = rgt; g < ngt; ++g) kept += fixw(sv_exp(__fsub_rn(gsv[g], M)));
    bs.flag = req2;
    bs.flag2 = rgt;
    bs.u64a = kept;
  }
  __syncthreads();
  const int req = bs.flag, rgt = bs.flag2;
  const uint64_t kept_tot = bs.u64a;
  const bool has_b = rgt < ngt;
  const uint64_t bkey = has_b ? (((uint64_t)ord_key(gsv[rgt]) << 32) | (uint32_t)gsi[rgt]) : ~0ull;
  const uint64_t Tu = MODE == MODE_SAMPLE ? mulfloor(kept_tot, u) : 0;
  const float Sf = fix_to_float(kept_tot);
  __syncthreads();
  if (tid == 0) bs.flag = -1;
  __syncthreads();

  // One index-ordered pass: tie ranks, kept positions, the draw, the outputs.
  int eq_before = 0, kept_before = 0;
  uint64_t w_before = 0;
  constexpr int Q = 4;
  for (int64_t base = 0; base < V; base += (int64_t)NT * Q) {
    float f[Q];
    bool iseq[Q], kept[Q];
    int neq_l = 0;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int64_t i = base + (int64_t)tid * Q + q;
      f[q] = i < V ? F(i) : NEG;
      iseq[q] = have_thr && f[q] > NEG && ord_key(f[q]) == K;
      neq_l += iseq[q];
    }
    int eq_tot;
    int eq_ex = block_excl_scan<NT, int>(neq_l, bs.iscr, &eq_tot);
    int kept_l = 0;
    uint64_t w_l = 0;
    uint64_t wq[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int64_t i = base + (int64_t)tid * Q + q;
      if (iseq[q]) {
        kept[q] = eq_before + eq_ex >= req;
        ++eq_ex;
      } else if (f[q] > NEG && (!have_thr || ord_key(f[q]) > K)) {
        kept[q] = (((uint64_t)ord_key(f[q]) << 32) | (uint32_t)i) >= bkey;
      } else {
        kept[q] = false;
      }
      wq[q] = kept[q] ? (iseq[q] ? Wt : fixw(sv_exp(__fsub_rn(f[q], M)))) : 0;
      kept_l += kept[q];
      w_l += wq[q];
    }
    int kept_tile;
    int kept_ex = block_excl_scan<NT, int>(kept_l, bs.iscr, &kept_tile);
    unsigned long long w_tile;
    unsigned long long w_ex = block_excl_scan<NT, unsigned long long>(w_l, bs.bsum, &w_tile);
    int pos = kept_before + kept_ex;
    uint64_t c = w_before + w_ex;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int64_t i = base + (int64_t)tid * Q + q;
      if (i >= V) break;
      if (kept[q]) {
        emit(pos, (int)i, f[q], Sf, M);
        ++pos;
        c += wq[q];
        if (MODE == MODE_SAMPLE && c > Tu && c - wq[q] <= Tu) bs.flag = (int)i;
      }
      if (a.out_dense && a.dense_mode != DENSE_NONE) {
        float dv;
        if (a.dense_mode == DENSE_SCORES) dv = kept[q] ? f[q] : NEG;
        else dv = kept[q] ? __fdiv_rn(sv_exp(__fsub_rn(f[q], M)), Sf) : 0.0f;
        a.out_dense[row * a.dense_stride + i] = dv;
      }
    }
    eq_before += eq_tot;
    kept_before += kept_tile;
    w_before += w_tile;
  }
  __syncthreads();
  if (MODE == MODE_SAMPLE) *token = bs.flag;
  Kept k;
  k.n = kept_before;
  k.M = M;
  k.tot = kept_tot;
  __syncthreads();
  return k;
}

// ------------------------------------------------- small-candidate finish

// Shared state of finish_small (the batched kernel lays it over its hit queues,
// which are dead by then; the vocab-sharded merge over its sorted list).
struct SmallFin {
  ulonglong2 kw[64];   // candidates: {(value key, index), weight}
  ulonglong2 kw2[64];  // kept entries: {index, weight}
  unsigned long long all, below, removed;
  float thr;
  int f0, r, hit, last;
};

// The finish of a row with m <= 64 candidates (fv, fi: tempered scores and
// indices) by the whole block, two threads per candidate: each pair finds its
// candidate's position and inclusive prefix sum in the ascending (value, index)
// order, then in the index order of the kept entries, each thread taking every
// other candidate and the pair adding their halves with one shuffle.  The k-th
// largest with ties (runtime_shared.py:180-181), top-p with `keep` (:182-186) and
// the index-order draw use the same exact integer arithmetic as warp_finish and
// leader_fast.  M is the largest candidate.  Returns the Kept summary, sets
// *token and writes the kept list in index order to kidx / kval (which may alias
// fi / fv).  Every thread of the block must call it.
template <int NT>
__device__ Kept finish_small(const RowArgs& a, const float* fv, const int* fi, int m, float M, float u,
                             int64_t* token, int* kidx, float* kval, SmallFin& f) {
  static_assert(NT >= 128, "two threads per candidate, 64 candidates");
  constexpr unsigned FULL = 0xffffffffu;
  const int tid = threadIdx.x;
  const int j = tid >> 1, h = tid & 1;
  const bool act = j < m;
  const float NEG = Elem<float>::neg_inf();
  float v = NEG;
  int id = 0;
  uint64_t key = ~0ull, e = 0;
  if (act) {
    v = fv[j];
    id = fi[j];
    key = ((uint64_t)ord_key(v) << 32) | (uint32_t)id;
    e = fixw(sv_exp(__fsub_rn(v, M)));
    if (h == 0) f.kw[j] = make_ulonglong2(key, e);
  }
  if (tid == 0) {
    f.below = 0;
    f.removed = 0;
    f.thr = NEG;
    f.f0 = 0;
    f.r = 0;
    f.hit = 0x7fffffff;
    f.last = -1;
  }
  __syncthreads();
  // Position and inclusive prefix sum in the ascending (value, index) order.
  int rk = 0;
  uint64_t S = 0;
  if (act) {
#pragma unroll 4
    for (int i = h; i < m; i += 2) {
      const ulonglong2 kw = f.kw[i];
      rk += kw.x < key;
      S += kw.x <= key ? kw.y : 0ull;
    }
  }
  rk += __shfl_xor_sync(FULL, rk, 1);
  S += __shfl_xor_sync(FULL, S, 1);
  if (act && h == 0) {
    if (m >= a.kk && rk == m - a.kk) f.thr = v;  // the k-th largest value
    if (rk == m - 1) f.all = S;                  // the largest holds the whole mass
  }
  __syncthreads();
  const float thr = f.thr;
  const bool in = act && v >= thr;  // ties with the k-th largest are kept
  if (act && h == 0 && !in) {
    atomicAdd(&f.f0, 1);
    atomicAdd(&f.below, (unsigned long long)e);
  }
  __syncthreads();
  const int f0 = f.f0, m1 = m - f0;
  const uint64_t below = f.below, total = f.all - below;
  // Top-p: the ascending prefix with mass <= floor(total * pthr) goes, never the
  // last `keep`.
  bool rm = false;
  if (a.pthr > 0.0f && in) {
    const uint64_t thrW = mulfloor(total, a.pthr);
    const int cap = m1 - a.keep > 0 ? m1 - a.keep : 0;
    rm = S - below <= thrW && rk - f0 < cap;
    if (rm && h == 0) {
      atomicAdd(&f.r, 1);
      atomicMax(&f.removed, (unsigned long long)(S - below));
    }
  }
  const bool q = in && !rm;
  if (act && h == 0) f.kw2[j] = make_ulonglong2(q ? (uint64_t)(uint32_t)id : ~0ull, q ? e : 0ull);
  __syncthreads();
  Kept kp;
  kp.n = m1 - f.r;
  kp.M = M;
  kp.tot = total - f.removed;
  // Position and inclusive prefix sum in index order over the kept entries; the
  // draw is the first index whose prefix exceeds floor(u * mass), else the last.
  int p = 0;
  uint64_t Q = 0;
  if (act) {
    const uint64_t ix = (uint32_t)id;
#pragma unroll 4
    for (int i = h; i < m; i += 2) {
      const ulonglong2 kw = f.kw2[i];
      p += kw.x < ix;
      Q += kw.x <= ix ? kw.y : 0ull;
    }
  }
  p += __shfl_xor_sync(FULL, p, 1);
  Q += __shfl_xor_sync(FULL, Q, 1);
  if (q && h == 0) {
    if (Q > mulfloor(kp.tot, u)) atomicMin(&f.hit, id);
    atomicMax(&f.last, id);
    kidx[p] = id;
    kval[p] = v;
  }
  __syncthreads();
  *token = f.hit != 0x7fffffff ? f.hit : f.last;
  return kp;
}

}  // namespace sv
