// sv_rows.cu -- the fused decode-sampling row kernel (sm_100a).
//
// One thread-block cluster of S CTAs per row (a row = one sequence in sample mode,
// one beam in beam mode).  CTA c of the cluster owns the vocabulary slice
// [c*slice_len, (c+1)*slice_len).  Per row:
//   0. TMA bulk copies (cp.async.bulk, mbarrier completion) stage the slice in
//      shared memory while the threads build the slice's seen-mask from the
//      history (ids, a byte mask or a bitmap).
//   1. Sample mode: repetition penalty (runtime_shared.py:172-173), written back
//      in place for fp32, and a NaN-propagating maximum per group of lanes.
//      Beam mode: the row maximum and the exact fixed-point sum of exp(x - M)
//      (log_softmax, runtime_shared.py:230), exchanged across the cluster through
//      distributed shared memory, and per-group maxima of seen / unseen logits.
//   2. The k-th largest of the kGroups group maxima is a lower bound tau of the
//      row's k-th largest penalised score (kGroups disjoint groups, k of them have
//      a maximum >= tau).  Every element >= tau (lowered by a margin that covers the
//      temperature rounding) is pushed, tempered, into the leader CTA's candidate
//      buffer through distributed shared memory.
//   3. The leader (cluster rank 0) finishes the row from the ~k candidates: exact
//      top-k threshold with ties (runtime_shared.py:180-181), top-p over the
//      ascending (value, index) order with exact fixed-point mass (:182-186), the
//      draw (sample mode) or the kept list for the beam merge (beam mode).
//      More than kCandCap candidates (huge tie groups) take a general path that
//      re-reads the row from global memory and handles the tie group
//      arithmetically.
//   4. Beam mode: the last beam leader to finish (atomic counter, no waiting)
//      merges the beams: + running scores, softmax over beams*V, count_nonzero,
//      draws without replacement (runtime_shared.py:231-237).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "sv_common.cuh"
#include "sv_internal.h"

namespace cg = cooperative_groups;

namespace sv {

constexpr int NT = kThreads;
constexpr int NWARP = NT / 32;
constexpr int CAP = kCandCap;

struct __align__(16) Shared {
  unsigned long long mbar[kChunks];
  float gmax[kGroups];
  float gmax2[kGroups];
  float red_max[kMaxCluster];
  unsigned long long red_sum[kMaxCluster];
  unsigned long long bsum[NWARP];
  float bmax[NWARP];
  int bint[NWARP];
  int cand_n;
  int err;
  int flag;
  int flag2;
  float tau_eff;
  float rowM, rowL;
  unsigned long long u64a, u64b;
  __align__(16) float cand_val[CAP];
  int cand_idx[CAP];
};

size_t shared_static_bytes() { return (sizeof(Shared) + 127) & ~size_t(127); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------- block helpers

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

__device__ uint64_t block_sum_u64(Shared& sh, uint64_t v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_u64(v);
  __syncthreads();
  if (lane == 0) sh.bsum[warp] = v;
  __syncthreads();
  uint64_t t = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) t += sh.bsum[w];
  return t;
}

__device__ int block_sum_int(Shared& sh, int v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_int(v);
  __syncthreads();
  if (lane == 0) sh.bint[warp] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) t += sh.bint[w];
  return t;
}

__device__ float block_max_nan(Shared& sh, float v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max_nan(v);
  __syncthreads();
  if (lane == 0) sh.bmax[warp] = v;
  __syncthreads();
  float t = sh.bmax[0];
#pragma unroll
  for (int w = 1; w < NWARP; ++w) t = max_nan(t, sh.bmax[w]);
  return t;
}

// Exclusive block scan of one value per thread; returns the prefix, *total the sum.
template <typename T>
__device__ T block_excl_scan(T v, T* scratch /* NWARP */, T* total) {
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
  for (int w = 0; w < NWARP; ++w) {
    T s = scratch[w];
    if (w < warp) before += s;
    all += s;
  }
  *total = all;
  return before + incl - v;
}

// In-place inclusive scan of a[0, n) (n <= NT * 4) by the whole block.
__device__ void block_scan_inplace_u64(Shared& sh, uint64_t* a, int n) {
  const int per = (n + NT - 1) / NT;
  const int b = threadIdx.x * per;
  uint64_t s = 0;
  for (int q = 0; q < per; ++q)
    if (b + q < n) { s += a[b + q]; a[b + q] = s; }
  uint64_t tot;
  uint64_t ex = block_excl_scan<unsigned long long>(s, sh.bsum, (unsigned long long*)&tot);
  for (int q = 0; q < per; ++q)
    if (b + q < n) a[b + q] += ex;
  __syncthreads();
}

// ------------------------------------------------------------ cluster helpers

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ T* remote(cg::cluster_group& cl, T* p, int rank) {
  return cl.map_shared_rank(p, rank);
}

// Bounded wait on an mbarrier phase: gives up after ~1 s of global time.
__device__ bool mbar_wait(uint32_t bar, uint32_t phase) {
  const uint64_t t0 = gtimer_ns();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(phase)
        : "memory");
    if (ok) return true;
    if (gtimer_ns() - t0 > 1000000000ull) return false;
  }
}

// ------------------------------------------------------------------ units
// A "unit" is 16 bytes of the staged slice: 4 fp32 or 8 fp16/bf16 values.

template <typename TIn> struct UnitIO;
template <> struct UnitIO<float> {
  static constexpr int E = 4;
  __device__ static void load(const float* d, int u, float (&v)[E]) {
    float4 t = reinterpret_cast<const float4*>(d)[u];
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  }
  __device__ static void store(float* d, int u, const float (&v)[E]) {
    reinterpret_cast<float4*>(d)[u] = make_float4(v[0], v[1], v[2], v[3]);
  }
  __device__ static uint32_t mask(const unsigned char* m, int u) {
    return reinterpret_cast<const uint32_t*>(m)[u];
  }
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
  __device__ static uint64_t mask(const unsigned char* m, int u) {
    return reinterpret_cast<const uint64_t*>(m)[u];
  }
};
template <> struct UnitIO<__half> : UnitIOHalf<__half> {};
template <> struct UnitIO<__nv_bfloat16> : UnitIOHalf<__nv_bfloat16> {};

__device__ __forceinline__ bool mask_bit(uint64_t m, int e) { return (m >> (8 * e)) & 0xffu; }

// History id access (int32 or int64 ids).
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

// Sets mask[id - lo] for the history ids in [lo, hi).  Loads are issued in batches
// of 8 per thread before any store, so their latencies overlap (the shared-memory
// stores could otherwise alias the loads and serialise them).  Returns the
// ST_HISTORY error bit for ids outside [0, V).
template <typename Id>
__device__ __forceinline__ int mark_ids(const Id* __restrict__ h, int64_t L, int64_t V, int64_t lo, int64_t hi,
                                        unsigned char* m) {
  constexpr int U = 8;
  int err = 0;
  for (int64_t base = 0; base < L; base += (int64_t)NT * U) {
    int64_t id[U];
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const int64_t j = base + threadIdx.x + (int64_t)q * NT;
      id[q] = j < L ? (int64_t)__ldg(h + j) : lo - 1;
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

// tau_eff: tau lowered by |tau| 2^-16 + T 2^-140 + 2^-140 (rounded towards -inf).
// Any element whose tempered value can equal the k-th largest tempered value is
// within T * ulp of the k-th largest penalised value, far inside this margin.
__device__ __forceinline__ float lower_tau(float tau, float T) {
  if (tau == Elem<float>::neg_inf()) return tau;
  float m = __fadd_ru(__fmul_ru(fabsf(tau), 1.52587890625e-05f), __fmul_ru(T, 7.174648137343064e-43f));
  m = __fadd_ru(m, 7.174648137343064e-43f);
  return __fsub_rd(tau, m);
}

// k-th largest (1-based, k <= kGroups) of the kGroups group maxima by warp 0;
// writes tau_eff (NaN-free) or an error code into sh.err.
__device__ void compute_tau(Shared& sh, const float* g, int kk, float T) {
  const int lane = threadIdx.x & 31;
  float v[4];
  uint32_t k4[4];
  bool nan = false, pinf = false;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = g[lane * 4 + q];
    nan |= v[q] != v[q];
    pinf |= v[q] == __int_as_float(0x7f800000);
    k4[q] = ord_key(v[q]);
  }
  nan = __any_sync(0xffffffffu, nan);
  pinf = __any_sync(0xffffffffu, pinf);
  uint32_t res = 0;
  for (int b = 31; b >= 0; --b) {
    uint32_t c = res | (1u << b);
    int n = __popc(__ballot_sync(0xffffffffu, k4[0] >= c)) + __popc(__ballot_sync(0xffffffffu, k4[1] >= c)) +
            __popc(__ballot_sync(0xffffffffu, k4[2] >= c)) + __popc(__ballot_sync(0xffffffffu, k4[3] >= c));
    if (n >= kk) res = c;
  }
  if (lane == 0) {
    if (nan) sh.err |= 1 << ST_NAN;
    else if (pinf) sh.err |= 1 << ST_POSINF;
    sh.tau_eff = lower_tau(key_to_float(res), T);
  }
}

__device__ __forceinline__ int first_err(int e) {
  for (int s = 1; s < 8; ++s)
    if (e & (1 << s)) return s;
  return ST_OK;
}

// ---------------------------------------------------------------- leader: fast
// Kept entries are returned in index order in (kidx, kval); count and the row max.
struct Kept {
  int n;          // kept count
  float M;        // row maximum of the warped scores
  uint64_t tot;   // fixed-point mass of the kept entries
};

// Top-k threshold, top-p and the index-ordered kept list from n <= CAP candidates.
__device__ Kept leader_fast(const RowArgs& a, Shared& sh, unsigned char* regA, int n, int* kidx, float* kval) {
  const int tid = threadIdx.x;
  float* sval = reinterpret_cast<float*>(regA);
  int* sidx = reinterpret_cast<int*>(regA + 4 * CAP);
  uint64_t* W = reinterpret_cast<uint64_t*>(regA + 8 * CAP);
  // (a) ascending order by (value, index): rank counting over ordered keys.
  for (int t = tid; t < n; t += NT)
    W[t] = ((uint64_t)ord_key(sh.cand_val[t]) << 32) | (uint32_t)sh.cand_idx[t];
  __syncthreads();
  for (int t = tid; t < n; t += NT) {
    const uint64_t kt = W[t];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += W[j] < kt;
    sval[rank] = sh.cand_val[t];
    sidx[rank] = sh.cand_idx[t];
  }
  __syncthreads();
  // (b) exact k-th largest with ties: survivors are sorted positions [f0, n).
  const int kk = a.kk;
  const float thr = n >= kk ? sval[n - kk] : Elem<float>::neg_inf();
  if (tid == 0) sh.flag = 0;
  __syncthreads();
  for (int j = tid; j < n; j += NT)
    if (sval[j] >= thr && (j == 0 || sval[j - 1] < thr)) sh.flag = j;
  __syncthreads();
  const int f0 = sh.flag;
  const int m = n - f0;
  const float M = sval[n - 1];
  // (c) weights
  for (int j = f0 + tid; j < n; j += NT) W[j] = fixw(sv_exp(__fsub_rn(sval[j], M)));
  __syncthreads();
  uint64_t lsum = 0;
  for (int j = f0 + tid; j < n; j += NT) lsum += W[j];
  const uint64_t total = block_sum_u64(sh, lsum);
  // (d) top-p: remove the ascending prefix whose mass is <= floor(total * pthr),
  //     never the last `keep` (runtime_shared.py:184-185).
  int r = 0;
  uint64_t removed = 0;
  if (a.pthr > 0.0f) {
    uint64_t* P = reinterpret_cast<uint64_t*>(sh.cand_val);  // candidates are consumed
    for (int j = tid; j < m; j += NT) P[j] = W[f0 + j];
    __syncthreads();
    block_scan_inplace_u64(sh, P, m);
    const uint64_t thrW = mulfloor(total, a.pthr);
    if (tid == 0) sh.flag = m;
    __syncthreads();
    for (int j = tid; j < m; j += NT)
      if (P[j] > thrW && (j == 0 || P[j - 1] <= thrW)) sh.flag = j;
    __syncthreads();
    r = sh.flag;
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

// ---------------------------------------------------------------- leader: slow
// General path over the whole row from global memory (huge tie groups, or forced).
// Writes the kept entries in index order through `emit(pos, idx, value)` and, in
// sample mode, draws the token.  Returns the kept count, row max and kept mass.
template <typename TIn, int MODE, typename Emit>
__device__ Kept leader_slow(const RowArgs& a, Shared& sh, unsigned char* regA, int64_t row, float bM, float bL,
                            float u, int64_t* token, Emit emit) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t V = a.vocab;
  const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
  const int nw = (int)((V + 31) >> 5);
  uint32_t* bits = reinterpret_cast<uint32_t*>(regA);
  unsigned char* rest = regA + ((size_t)nw * 4 + 127) / 128 * 128;
  uint32_t* hist = reinterpret_cast<uint32_t*>(rest);        // 256 bins
  float* gval = reinterpret_cast<float*>(rest + 1024);        // <= kMaxTopK
  int* gidx = reinterpret_cast<int*>(rest + 1024 + 4 * kMaxTopK);
  float* gsv = reinterpret_cast<float*>(rest + 1024 + 8 * kMaxTopK);
  int* gsi = reinterpret_cast<int*>(rest + 1024 + 12 * kMaxTopK);
  uint64_t* scr = reinterpret_cast<uint64_t*>(rest + 1024 + 16 * kMaxTopK);  // NWARP
  int* iscr = reinterpret_cast<int*>(rest + 1024 + 16 * kMaxTopK + 8 * NWARP);

  // Seen bitmap of the whole row.
  for (int w = tid; w < nw; w += NT) bits[w] = 0;
  __syncthreads();
  if (a.hist_kind == HIST_IDS32 || a.hist_kind == HIST_IDS64) {
    const int64_t L = hist_length(a, row);
    for (int64_t j = tid; j < L; j += NT) {
      const int64_t id = hist_id(a, row, j);
      if (id >= 0 && id < V) atomicOr(&bits[id >> 5], 1u << (id & 31));
    }
  } else if (a.hist_kind == HIST_MASK8 || a.hist_kind == HIST_BITS32) {
    for (int64_t i = tid; i < V; i += NT)
      if (seen_global(a, row, i)) atomicOr(&bits[i >> 5], 1u << (i & 31));
  }
  __syncthreads();
  const float rp = a.rep_penalty, T = a.temperature;
  auto F = [&](int64_t i) -> float {
    float x = Elem<TIn>::load(rowp + i);
    if (MODE == MODE_BEAM) x = __fsub_rn(__fsub_rn(x, bM), bL);
    if ((bits[i >> 5] >> (i & 31)) & 1u) x = penalize(x, rp);
    return temper(x, T);
  };
  const float NEG = Elem<float>::neg_inf();
  const int kk = a.kk;

  // Exact k-th largest key K by 8-bit radix select over finite values.
  int nfin = 0;
  for (int64_t i = tid; i < V; i += NT) nfin += F(i) > NEG;
  nfin = block_sum_int(sh, nfin);
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
        for (int q = 0; q < 8; ++q) { c[q] = hist[lane * 8 + q]; s += c[q]; }
        uint32_t incl = s;  // sum over lanes >= lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
          if (lane + o < 32) incl += t;
        }
        if (incl >= (uint32_t)need && incl - s < (uint32_t)need) {
          uint32_t above = incl - s;
          for (int q = 7; q >= 0; --q) {
            if (above + c[q] >= (uint32_t)need) { sh.flag = lane * 8 + q; sh.flag2 = (int)above; break; }
            above += c[q];
          }
        }
      }
      __syncthreads();
      prefix |= (uint32_t)sh.flag << shf;
      pmask |= 255u << shf;
      need -= sh.flag2;
      __syncthreads();
    }
  }
  const uint32_t K = prefix;
  const float thr = have_thr ? key_to_float(K) : NEG;

  // Count the tie group (key == K) and collect the entries above it (< kk).
  if (tid == 0) sh.flag = 0;
  __syncthreads();
  int neq = 0;
  for (int64_t i = tid; i < V; i += NT) {
    const float f = F(i);
    if (!(f > NEG)) continue;
    const uint32_t k = ord_key(f);
    if (have_thr && k == K) ++neq;
    else if (!have_thr || k > K) {
      const int s = atomicAdd(&sh.flag, 1);
      if (s < kMaxTopK) { gval[s] = f; gidx[s] = (int)i; }
    }
  }
  neq = block_sum_int(sh, neq);
  const int ngt = min(sh.flag, kMaxTopK);
  __syncthreads();
  // Sort the entries above the tie group ascending by (value, index).
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
      uint64_t req = Wt == 0 ? (uint64_t)neq : thrW / Wt;
      r = req < (uint64_t)neq ? (int)req : neq;
      if (r == neq) {
        uint64_t P = (uint64_t)neq * Wt;
        for (int g = 0; g < ngt; ++g) {
          P += fixw(sv_exp(__fsub_rn(gsv[g], M)));
          if (P <= thrW) ++r; else break;
        }
      }
      const int cap = m - a.keep > 0 ? m - a.keep : 0;
      if (r > cap) r = cap;
    }
    const int req = r < neq ? r : neq;
    const int rgt = r - req;
    uint64_t kept = (uint64_t)(neq - req) * Wt;
    for (int g = rgt; g < ngt; ++g) kept += fixw(sv_exp(__fsub_rn(gsv[g], M)));
    sh.flag = req;
    sh.flag2 = rgt;
    sh.u64a = kept;
  }
  __syncthreads();
  const int req = sh.flag, rgt = sh.flag2;
  const uint64_t kept_tot = sh.u64a;
  const bool has_b = rgt < ngt;
  const uint64_t bkey = has_b ? (((uint64_t)ord_key(gsv[rgt]) << 32) | (uint32_t)gsi[rgt]) : ~0ull;
  const uint64_t Tu = MODE == MODE_SAMPLE ? mulfloor(kept_tot, u) : 0;
  const float Sf = fix_to_float(kept_tot);
  __syncthreads();

  // One index-ordered pass: tie ranks, kept positions, the draw and the outputs.
  int eq_before = 0, kept_before = 0;
  uint64_t w_before = 0;
  if (tid == 0) sh.flag = -1;
  __syncthreads();
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
    int eq_ex = block_excl_scan<int>(neq_l, iscr, &eq_tot);
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
    int kept_tot_tile;
    int kept_ex = block_excl_scan<int>(kept_l, iscr, &kept_tot_tile);
    unsigned long long w_tot_tile;
    unsigned long long w_ex = block_excl_scan<unsigned long long>(w_l, (unsigned long long*)scr, &w_tot_tile);
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
        if (MODE == MODE_SAMPLE && c > Tu && c - wq[q] <= Tu) sh.flag = (int)i;
      }
      if (a.out_dense && a.dense_mode != DENSE_NONE) {
        float dv;
        if (a.dense_mode == DENSE_SCORES) dv = kept[q] ? f[q] : NEG;
        else dv = kept[q] ? __fdiv_rn(sv_exp(__fsub_rn(f[q], M)), Sf) : 0.0f;
        a.out_dense[row * a.dense_stride + i] = dv;
      }
    }
    eq_before += eq_tot;
    kept_before += kept_tot_tile;
    w_before += w_tot_tile;
  }
  __syncthreads();
  if (MODE == MODE_SAMPLE) *token = sh.flag;
  Kept k;
  k.n = kept_before;
  k.M = M;
  k.tot = kept_tot;
  __syncthreads();
  return k;
}

// ------------------------------------------------------------------ beam merge
// Runs in the last beam leader to finish.  Entries of all beams in flattened
// (beam-major, index-ascending) order; weights in `W` (shared or global).
__device__ void beam_merge(const RowArgs& a, Shared& sh, unsigned char* regA) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int B = a.rows;
  const BeamWsHeader* hdr = reinterpret_cast<const BeamWsHeader*>(a.ws);
  const int* kidx0 = reinterpret_cast<const int*>(a.ws + sizeof(BeamWsHeader));
  const float* kval0 = reinterpret_cast<const float*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 4);
  uint64_t* Wg = reinterpret_cast<uint64_t*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 8);
  __shared__ int offs[kMaxBeams + 1];
  __shared__ int picked[2 * kMaxBeams];
  if (tid == 0) {
    int st = ST_OK, o = 0;
    for (int b = 0; b < B; ++b) {
      const int s = __ldcg(&hdr->status[b]);
      if (s != ST_OK && st == ST_OK) st = s;
      offs[b] = o;
      o += __ldcg(&hdr->count[b]);
    }
    offs[B] = o;
    sh.flag = st;
  }
  __syncthreads();
  const int st = sh.flag;
  const int K = offs[B];
  if (st != ST_OK || K == 0) {
    if (tid == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = st != ST_OK ? st : ST_ALLNEGINF;
    }
    return;
  }
  auto beam_of = [&](int e) {
    int b = 0;
    while (offs[b + 1] <= e) ++b;
    return b;
  };
  auto score_of = [&](int e, int b) -> float {
    return __fadd_rn(__ldcg(&kval0[(size_t)b * a.ws_cap + (e - offs[b])]), a.running[b]);
  };
  // M* and the fixed-point total.
  float mx = Elem<float>::neg_inf();
  for (int e = tid; e < K; e += NT) mx = max_nan(mx, score_of(e, beam_of(e)));
  const float Ms = block_max_nan(sh, mx);
  const bool in_smem = K <= 2048;
  uint64_t* W = in_smem ? reinterpret_cast<uint64_t*>(regA) : Wg;
  uint64_t ls = 0;
  for (int e = tid; e < K; e += NT) {
    const float s = score_of(e, beam_of(e));
    W[e] = fixw(sv_exp(__fsub_rn(s, Ms)));
    ls += W[e];
  }
  const uint64_t tot = block_sum_u64(sh, ls);
  const float Sf = fix_to_float(tot);
  int nz = 0;
  for (int e = tid; e < K; e += NT) {
    const int b = beam_of(e);
    const float p = __fdiv_rn(sv_exp(__fsub_rn(score_of(e, b), Ms)), Sf);
    nz += p > 0.0f;
    const int j = e - offs[b];
    if (a.out_prob && j < a.out_cap) a.out_prob[(size_t)b * a.out_cap + j] = p;
  }
  const int nnz = block_sum_int(sh, nz);
  const int n = a.npick < nnz ? a.npick : nnz;
  __syncthreads();
  if (tid < 32) {
    const int seg = (K + 31) / 32;
    const int e0 = lane * seg, e1 = min(K, e0 + seg);
    uint64_t mysum = 0;
    for (int e = e0; e < e1; ++e) mysum += W[e];
    for (int j = 0; j < n; ++j) {
      const uint64_t total = warp_sum_u64(mysum);
      int pick = -1;
      if (total > 0) {
        const uint64_t t = mulfloor(total, a.uniforms[j]);
        uint64_t incl = mysum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          uint64_t v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const uint64_t excl = incl - mysum;
        const bool own = mysum > 0 && excl <= t && t < incl;
        const unsigned bm = __ballot_sync(0xffffffffu, own);
        const int o = __ffs(bm) - 1;
        if (lane == o) {
          uint64_t c = excl;
          for (int e = e0; e < e1; ++e) {
            c += W[e];
            if (c > t) { pick = e; break; }
          }
          mysum -= W[pick];
          W[pick] = 0;
        }
        pick = __shfl_sync(0xffffffffu, pick, o);
      } else {
        // No fixed-point mass left: the largest remaining nonzero probability.
        float best = -1.0f;
        int be = K;
        for (int e = e0; e < e1; ++e) {
          bool done = false;
          for (int q = 0; q < j; ++q) done |= picked[q] == e;
          if (done) continue;
          const float p = __fdiv_rn(sv_exp(__fsub_rn(score_of(e, beam_of(e)), Ms)), Sf);
          if (p > 0.0f && (p > best || (p == best && e < be))) { best = p; be = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          float ob = __shfl_xor_sync(0xffffffffu, best, o);
          int oe = __shfl_xor_sync(0xffffffffu, be, o);
          if (ob > best || (ob == best && oe < be)) { best = ob; be = oe; }
        }
        pick = be;
      }
      if (lane == 0) {
        picked[j] = pick;
        const int b = beam_of(pick);
        a.out_picks[j] = (int64_t)b * a.vocab + __ldcg(&kidx0[(size_t)b * a.ws_cap + (pick - offs[b])]);
        a.out_pick_scores[j] = score_of(pick, b);
      }
      __syncwarp();
    }
    if (lane == 0) {
      *a.out_npicks = n;
      a.out_status[0] = ST_OK;
    }
  }
}

// ------------------------------------------------------------------ the kernel

template <typename TIn, int MODE>
__global__ void __launch_bounds__(NT, 3) row_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>(smem_raw);
  unsigned char* regA = smem_raw + ((sizeof(Shared) + 127) & ~size_t(127));
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int ES = Elem<TIn>::kSize;
  constexpr int EPU = 16 / ES;
  using IO = UnitIO<TIn>;
  const int S = a.S;
  const int crank = (int)cluster.block_rank();
  const int64_t row = blockIdx.x / S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float NEG = Elem<float>::neg_inf();

  cluster_arrive_relaxed();  // completes before the first remote access

  const int64_t V = a.vocab;
  const int64_t lo = (int64_t)crank * a.slice_len;
  const int64_t hi = min(V, lo + (int64_t)a.slice_len);
  const int64_t nel = hi > lo ? hi - lo : 0;
  const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
  const uintptr_t gs = reinterpret_cast<uintptr_t>(rowp + lo);
  const uintptr_t ge = gs + (uintptr_t)nel * ES;
  const uintptr_t base16 = gs & ~uintptr_t(15);
  const int off_e = (int)((gs - base16) / ES);
  const int nunits = nel ? (int)((ge - base16 + 15) / 16) : 0;
  const int npos = nunits * EPU;
  TIn* data = reinterpret_cast<TIn*>(regA);
  unsigned char* mask = regA + (((size_t)a.slice_len * ES + 32 + 127) & ~size_t(127));

  const uintptr_t b_lo = (gs + 15) & ~uintptr_t(15);
  const uintptr_t b_hi = ge & ~uintptr_t(15);
  const bool has_bulk = nel > 0 && b_hi > b_lo;
  const uint32_t bulk_bytes = has_bulk ? (uint32_t)(b_hi - b_lo) : 0;
  const uint32_t csz = ((bulk_bytes + kChunks - 1) / kChunks + 15) & ~15u;

  if (tid == 0) {
    sh.cand_n = 0;
    sh.err = 0;
#pragma unroll
    for (int c = 0; c < kChunks; ++c)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sh.mbar[c])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && has_bulk) {
    unsigned char* dst = reinterpret_cast<unsigned char*>(data) + (b_lo - base16);
    for (int c = 0; c < kChunks; ++c) {
      const uint32_t off = (uint32_t)c * csz;
      if (off >= bulk_bytes) break;
      const uint32_t sz = min(csz, bulk_bytes - off);
      const uint32_t bar = smem_u32(&sh.mbar[c]);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(sz) : "memory");
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(dst + off)),
          "l"(reinterpret_cast<const void*>(b_lo + off)), "r"(sz), "r"(bar)
          : "memory");
    }
  }
  // Ragged head / tail positions (outside the 16-byte-aligned bulk range) and the
  // -inf padding of the window.
  {
    const int ph_end = has_bulk ? (int)((b_lo - base16) / ES) : npos;
    const int pt_beg = has_bulk ? (int)((b_hi - base16) / ES) : npos;
    for (int p = tid; p < ph_end + (npos - pt_beg); p += NT) {
      const int pos = p < ph_end ? p : pt_beg + (p - ph_end);
      const int64_t e = pos - off_e;
      data[pos] = (e >= 0 && e < nel) ? __ldg(rowp + lo + e) : Elem<TIn>::neg_inf();
    }
  }
  // Seen mask of the window.
  const int mbytes = (npos + 15) & ~15;
  for (int p = tid * 16; p < mbytes; p += NT * 16) *reinterpret_cast<uint4*>(mask + p) = make_uint4(0, 0, 0, 0);
  __syncthreads();
  int local_err = 0;
  if (a.hist_kind == HIST_IDS32) {
    local_err |= mark_ids(reinterpret_cast<const int32_t*>(a.hist) + row * a.hist_stride, hist_length(a, row), V,
                          lo, hi, mask + off_e);
  } else if (a.hist_kind == HIST_IDS64) {
    local_err |= mark_ids(reinterpret_cast<const int64_t*>(a.hist) + row * a.hist_stride, hist_length(a, row), V,
                          lo, hi, mask + off_e);
  } else if (a.hist_kind == HIST_MASK8 || a.hist_kind == HIST_BITS32) {
    for (int64_t e = tid; e < nel; e += NT) mask[off_e + e] = seen_global(a, row, lo + e);
  }
  __syncthreads();

  // Wait for the bulk chunks (bounded).
  bool timeout = false;
  if (has_bulk) {
    for (int c = 0; c < kChunks; ++c) {
      if ((uint32_t)c * csz >= bulk_bytes) break;
      if (!mbar_wait(smem_u32(&sh.mbar[c]), 0)) timeout = true;
    }
  }
  if (timeout) local_err |= 1 << ST_TIMEOUT;

  const float rp = a.rep_penalty, T = a.temperature;
  const int GS = 2 * S;  // lanes per group: kGroups = S * NT / GS
  const int g = crank * (NT / GS) + tid / GS;
  float bM = 0.0f, bL = 0.0f;

  if (MODE == MODE_SAMPLE) {
    // Pass 1: penalty (in place for fp32) and group maxima.
    float tmax = NEG;
    for (int u = tid; u < nunits; u += NT) {
      float v[EPU];
      IO::load(data, u, v);
      const uint64_t mk = (uint64_t)IO::mask(mask, u);
#pragma unroll
      for (int e = 0; e < EPU; ++e) {
        if (mask_bit(mk, e)) v[e] = penalize(v[e], rp);
        tmax = max_nan(tmax, v[e]);
      }
      if (ES == 4 && mk) IO::store(data, u, v);
    }
    for (int o = 1; o < GS; o <<= 1) tmax = max_nan(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    cluster_wait();
    if (tid % GS == 0)
      for (int r = 0; r < S; ++r) *remote(cluster, &sh.gmax[g], r) = tmax;
    if (local_err) atomicOr(remote(cluster, &sh.err, 0), local_err);
    cluster_sync_all();  // #1
    if (warp == 0) compute_tau(sh, sh.gmax, a.kk, T);
    __syncthreads();
  } else {
    // Beam pass A: row maximum.
    float tmax = NEG;
    for (int u = tid; u < nunits; u += NT) {
      float v[EPU];
      IO::load(data, u, v);
#pragma unroll
      for (int e = 0; e < EPU; ++e) tmax = max_nan(tmax, v[e]);
    }
    tmax = block_max_nan(sh, tmax);
    cluster_wait();
    if (tid < S) *remote(cluster, &sh.red_max[crank], tid) = tmax;
    if (local_err) atomicOr(remote(cluster, &sh.err, 0), local_err);
    cluster_sync_all();  // #A
    float M = sh.red_max[0];
    for (int r = 1; r < S; ++r) M = max_nan(M, sh.red_max[r]);
    const bool bad = M != M || M == __int_as_float(0x7f800000) || M == NEG;
    // Beam pass B: fixed-point sum of exp(x - M), seen / unseen group maxima.
    uint64_t lsum = 0;
    float gu = NEG, gsn = NEG;
    if (!bad) {
      for (int u = tid; u < nunits; u += NT) {
        float v[EPU];
        IO::load(data, u, v);
        const uint64_t mk = (uint64_t)IO::mask(mask, u);
#pragma unroll
        for (int e = 0; e < EPU; ++e) {
          lsum += fixw(sv_exp(__fsub_rn(v[e], M)));
          if (mask_bit(mk, e)) gsn = fmaxf(gsn, v[e]);
          else gu = fmaxf(gu, v[e]);
        }
      }
    }
    lsum = block_sum_u64(sh, lsum);
    for (int o = 1; o < GS; o <<= 1) {
      gu = fmaxf(gu, __shfl_xor_sync(0xffffffffu, gu, o));
      gsn = fmaxf(gsn, __shfl_xor_sync(0xffffffffu, gsn, o));
    }
    if (tid < S) *remote(cluster, &sh.red_sum[crank], tid) = lsum;
    if (tid % GS == 0)
      for (int r = 0; r < S; ++r) {
        *remote(cluster, &sh.gmax[g], r) = gu;
        *remote(cluster, &sh.gmax2[g], r) = gsn;
      }
    cluster_sync_all();  // #B
    uint64_t Ssum = 0;
    for (int r = 0; r < S; ++r) Ssum += sh.red_sum[r];
    bM = M;
    bL = bad ? 0.0f : log_fixed(Ssum);
    // Group maxima of the penalised log-probs: both maps are monotone.
    for (int q = tid; q < kGroups; q += NT) {
      const float fu = __fsub_rn(__fsub_rn(sh.gmax[q], bM), bL);
      const float fs = penalize(__fsub_rn(__fsub_rn(sh.gmax2[q], bM), bL), rp);
      sh.gmax[q] = fmaxf(fu, fs);
    }
    __syncthreads();
    if (warp == 0) {
      if (!bad) {
        compute_tau(sh, sh.gmax, a.kk, T);
      } else if (lane == 0) {
        sh.err |= 1 << (M != M ? ST_NAN : (M == NEG ? ST_ALLNEGINF : ST_POSINF));
        sh.tau_eff = __int_as_float(0x7fc00000);
      }
    }
    __syncthreads();
  }

  // Pass 2: push candidates >= tau_eff into the leader's buffer.
  const float te = sh.tau_eff;
  int* rcount = remote(cluster, &sh.cand_n, 0);
  float* rval = remote(cluster, sh.cand_val, 0);
  int* ridx = remote(cluster, sh.cand_idx, 0);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int ub = 0; ub < nunits; ub += NT) {
    const int u = ub + tid;
    float v[EPU];
    bool pass[EPU];
    bool any = false;
    if (u < nunits) {
      IO::load(data, u, v);
      if (MODE == MODE_BEAM || ES != 4) {
        const uint64_t mk = (uint64_t)IO::mask(mask, u);
#pragma unroll
        for (int e = 0; e < EPU; ++e) {
          if (MODE == MODE_BEAM) v[e] = __fsub_rn(__fsub_rn(v[e], bM), bL);
          if (mask_bit(mk, e)) v[e] = penalize(v[e], rp);
        }
      }
#pragma unroll
      for (int e = 0; e < EPU; ++e) {
        pass[e] = v[e] >= te && v[e] > NEG;
        any |= pass[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < EPU; ++e) pass[e] = false;
    }
    if (!__any_sync(0xffffffffu, any)) continue;
#pragma unroll
    for (int e = 0; e < EPU; ++e) {
      const unsigned bm = __ballot_sync(0xffffffffu, pass[e]);
      if (!bm) continue;
      const int ll = __ffs(bm) - 1;
      int base = 0;
      if (lane == ll) base = atomicAdd(rcount, __popc(bm));
      base = __shfl_sync(0xffffffffu, base, ll);
      if (pass[e]) {
        const int slot = base + __popc(bm & lt_mask);
        if (slot < CAP) {
          rval[slot] = temper(v[e], T);
          ridx[slot] = (int)(lo + (int64_t)(u * EPU + e) - off_e);
        }
      }
    }
  }
  if (a.out_dense && a.dense_mode != DENSE_NONE) {
    const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
    for (int64_t e = tid; e < nel; e += NT) a.out_dense[row * a.dense_stride + lo + e] = dv;
    __threadfence();
  }
  cluster_sync_all();  // #2: candidates complete; no remote access after this
  if (crank != 0) return;

  // ---------------------------------------------------------------- leader
  const int err = sh.err;
  int* kidx;
  float* kval;
  if (MODE == MODE_BEAM) {
    kidx = reinterpret_cast<int*>(a.ws + sizeof(BeamWsHeader)) + row * a.ws_cap;
    kval = reinterpret_cast<float*>(a.ws + sizeof(BeamWsHeader) + (size_t)a.rows * a.ws_cap * 4) + row * a.ws_cap;
  } else {
    kidx = sh.cand_idx;
    kval = sh.cand_val;
  }
  const float uu = MODE == MODE_SAMPLE ? a.uniforms[row] : 0.0f;
  int status = err ? first_err(err) : ST_OK;
  Kept kept = {0, 0.0f, 0};
  int64_t token = -1;
  const int n = sh.cand_n;
  // The row maximum is always a candidate when it is finite (tau <= max).
  if (status == ST_OK && n == 0) status = ST_ALLNEGINF;
  if (status == ST_OK) {
    if (!a.force_slow && n <= CAP) {
      kept = leader_fast(a, sh, regA, n, kidx, kval);
      const float Sf = fix_to_float(kept.tot);
      if (MODE == MODE_SAMPLE) {
        // Draw: index-ordered prefix of the kept weights against floor(u * total).
        uint64_t* Wk = reinterpret_cast<uint64_t*>(regA);
        for (int j = tid; j < kept.n; j += NT) Wk[j] = fixw(sv_exp(__fsub_rn(kval[j], kept.M)));
        __syncthreads();
        block_scan_inplace_u64(sh, Wk, kept.n);
        const uint64_t Tu = mulfloor(kept.tot, uu);
        if (tid == 0) sh.flag = kept.n - 1;
        __syncthreads();
        for (int j = tid; j < kept.n; j += NT)
          if (Wk[j] > Tu && (j == 0 || Wk[j - 1] <= Tu)) sh.flag = j;
        __syncthreads();
        token = kidx[sh.flag];
      }
      for (int j = tid; j < kept.n; j += NT) {
        const float p = __fdiv_rn(sv_exp(__fsub_rn(kval[j], kept.M)), Sf);
        if (j < a.out_cap) {
          if (a.out_idx) a.out_idx[row * a.out_cap + j] = kidx[j];
          if (MODE == MODE_SAMPLE && a.out_prob) a.out_prob[row * a.out_cap + j] = p;
          if (a.out_score) a.out_score[row * a.out_cap + j] = kval[j];
        }
        if (a.out_dense && a.dense_mode != DENSE_NONE)
          a.out_dense[row * a.dense_stride + kidx[j]] = a.dense_mode == DENSE_SCORES ? kval[j] : p;
      }
    } else {
      auto emit = [&](int pos, int idx, float val, float Sf, float M) {
        if (MODE == MODE_BEAM) {
          kidx[pos] = idx;
          kval[pos] = val;
        }
        if (pos < a.out_cap) {
          if (a.out_idx) a.out_idx[row * a.out_cap + pos] = idx;
          if (MODE == MODE_SAMPLE && a.out_prob)
            a.out_prob[row * a.out_cap + pos] = __fdiv_rn(sv_exp(__fsub_rn(val, M)), Sf);
          if (a.out_score) a.out_score[row * a.out_cap + pos] = val;
        }
      };
      kept = leader_slow<TIn, MODE>(a, sh, regA, row, bM, bL, uu, &token, emit);
    }
  }
  if (MODE == MODE_SAMPLE) {
    if (tid == 0) {
      a.out_token[row] = status == ST_OK ? token : -1;
      if (a.out_count) a.out_count[row] = kept.n;
      if (a.out_status) a.out_status[row] = status;
      if (status == ST_OK && a.seen_bits && token >= 0)
        atomicOr(&a.seen_bits[row * a.seen_bits_stride + (token >> 5)], 1u << (token & 31));
    }
    return;
  }
  // Beam: publish this beam's kept list, then the last leader merges.
  BeamWsHeader* hdr = reinterpret_cast<BeamWsHeader*>(a.ws);
  if (tid == 0) {
    hdr->status[row] = status;
    hdr->count[row] = kept.n;
    if (a.out_count) a.out_count[row] = kept.n;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sh.flag = atomicAdd(&hdr->counter, 1u) == (unsigned)(a.rows - 1);
  __syncthreads();
  if (!sh.flag) return;
  __threadfence();
  beam_merge(a, sh, regA);
  __syncthreads();
  if (tid == 0) atomicExch(&hdr->counter, 0u);
}

// ---------------------------------------------------------------- host launch

template <typename TIn, int MODE>
static cudaError_t launch_t(const RowArgs& a, size_t smem, cudaStream_t stream) {
  auto kern = row_kernel<TIn, MODE>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  static int max_dyn[64] = {0};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    max_dyn[dev] = optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn[dev]);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  if ((int64_t)smem > (int64_t)max_dyn[dev]) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.rows * a.S), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_rows(const RowArgs& a, size_t smem, cudaStream_t stream) {
  if (a.mode == MODE_SAMPLE) {
    if (a.dtype == DT_F32) return launch_t<float, MODE_SAMPLE>(a, smem, stream);
    if (a.dtype == DT_F16) return launch_t<__half, MODE_SAMPLE>(a, smem, stream);
    return launch_t<__nv_bfloat16, MODE_SAMPLE>(a, smem, stream);
  }
  if (a.dtype == DT_F32) return launch_t<float, MODE_BEAM>(a, smem, stream);
  if (a.dtype == DT_F16) return launch_t<__half, MODE_BEAM>(a, smem, stream);
  return launch_t<__nv_bfloat16, MODE_BEAM>(a, smem, stream);
}

}  // namespace sv
