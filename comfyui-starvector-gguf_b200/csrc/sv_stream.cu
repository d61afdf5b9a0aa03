// sv_stream.cu -- the batched row kernel (sm_100a): many independent rows.
//
// One CTA per row.  The row's logits stream straight into registers as 32-byte
// units (256-bit non-caching loads; one unit per thread per batch, the CTA's batch
// a contiguous NT*32-byte span) through a ring of RING register buffers, so
// RING - 1 batches are in flight while a warp works on one.  The logits are not
// staged in shared memory and no block barrier separates the batches.
//
// Per row (runtime_shared.py:200-202):
//   1. the row's seen bitmap in shared memory, from the history (its ids fetched
//      by one bulk copy issued as the CTA starts);
//   2. a first lower bound tau of the row's k-th largest penalised score: the
//      exact k-th largest of the threads' maxima over the unseen elements of the
//      first RING batches (NT distinct elements, each at or below its penalised
//      score);
//   3. every batch: the unit maxima of the raw scores (the penalty never raises a
//      score, so a unit below tau holds no candidate) and, for the rare units that
//      reach tau, each element's penalised score (:172-173, the seen bit looked up
//      only here).  Those reaching tau are appended to the warp's own candidate
//      list (ballot-aggregated, no shared counter) and counted in a 256-bin
//      histogram over ordered float keys shared by the CTA.  A warp whose list grew
//      by RW entries recomputes the bound from the histogram (the highest bin edge
//      with at least k counted values at or above it: counts only grow, so any
//      snapshot gives a valid bound) and raises the shared tau;
//   4. finish: the candidates reaching the final bound, tempered (:178-179); the
//      exact k-th largest with ties (:180-181), top-p over the ascending (value,
//      index) order with exact fixed-point mass (:182-186) and the draw from the
//      row's uniform, by one warp for up to 64 candidates (a block finish up to
//      256, the general path over the whole row beyond).  A row whose candidate
//      lists overflow is read again against the final bound.
// Status: a NaN anywhere in the row, else a +inf tempered score, else no finite
// score.  No inter-CTA communication and no scratch memory in global memory.
#include <cuda_runtime.h>

#include <type_traits>

#include "sv_block.cuh"
#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

namespace {

constexpr int UB = 32;       // bytes per unit (one 256-bit load)
constexpr int BU = 1;        // units per thread per batch
constexpr int RING = 4;      // batches in registers (RING - 1 in flight while one is worked on)
constexpr int QCAP = 32;     // queued hit units per warp
constexpr int CAP = 1024;    // candidate capacity per row (split evenly between the warps)
constexpr int SFIN = 256;    // candidates the fast finishes take
constexpr int SBINS = 256;   // bound histogram bins
constexpr int RW = 8;        // growth of a warp's list between its bound recomputations

// Bytes of the staging region: the row's history ids (bulk copy) at the start,
// then the candidate lists, the hit queues and the finish input.
__host__ __device__ constexpr int lists_bytes(int nt) {
  return 8 * CAP + (nt / 32) * QCAP * 36 + 8 * SFIN;
}
constexpr int kIdStage = 16 * 1024;  // history bytes taken by one bulk copy
__host__ __device__ constexpr int stage_bytes(int nt) {
  return lists_bytes(nt) > kIdStage ? lists_bytes(nt) : kIdStage;
}

template <int NT>
struct __align__(128) StreamShared {
  static constexpr int NW = NT / 32;
  BlockScratch<NT> bs;
  __align__(16) unsigned int bins[SBINS];
  float wsort[NW][32];  // first bound: each warp's values, descending
  int wcount[NW];       // candidates each warp found
  unsigned int tau_key;   // ordered key of the shared bound (atomicMax)
  unsigned int rmax_key;  // ordered key of the row's largest raw score
  int err;
  int ccount[NW];              // candidates of each warp's list reaching the final bound
  unsigned int mkey;           // ordered key of the largest tempered candidate
  unsigned long long idbar;  // completion of the history bulk copy
  __align__(128) unsigned char stage[stage_bytes(NT)];
  // The lists, over the staging region once the history is marked: candidates
  // (penalised score, index; warp w owns [w * CAP / NW, (w + 1) * CAP / NW)), each
  // warp's queued hit units (32 bytes each) and their unit numbers, the finish input.
  __device__ float* cval() { return reinterpret_cast<float*>(stage); }
  __device__ int* cidx() { return reinterpret_cast<int*>(stage + 4 * CAP); }
  __device__ uint4* qdata(int w) { return reinterpret_cast<uint4*>(stage + 8 * CAP) + w * 2 * QCAP; }
  __device__ int* qunit(int w) { return reinterpret_cast<int*>(stage + 8 * CAP + NW * QCAP * 32) + w * QCAP; }
  __device__ float* fv() { return reinterpret_cast<float*>(stage + 8 * CAP + NW * QCAP * 36); }
  __device__ int* fi() { return reinterpret_cast<int*>(stage + 8 * CAP + NW * QCAP * 36 + 4 * SFIN); }
};

__host__ __device__ constexpr size_t static_bytes(int nt) {
  return nt == 128 ? (sizeof(StreamShared<128>) + 127) & ~size_t(127)
         : nt == 256 ? (sizeof(StreamShared<256>) + 127) & ~size_t(127)
                     : (sizeof(StreamShared<512>) + 127) & ~size_t(127);
}

__host__ __device__ inline size_t bitmap_bytes(int64_t V) {
  return (((size_t)V + 31) / 32 * 4 + 16 + 127) & ~size_t(127);
}

// A 32-byte unit in registers: 8 fp32 or 16 fp16/bf16 values.
template <typename TIn> struct Unit;
template <> struct Unit<float> {
  static constexpr int E = 8;
  __device__ static float at(const uint32_t (&w)[8], int e) { return __uint_as_float(w[e]); }
  __device__ static void put(uint32_t (&w)[8], int e, float v) { w[e] = __float_as_uint(v); }
};
__device__ __forceinline__ void put16(uint32_t (&w)[8], int e, uint32_t b) {
  w[e >> 1] = (e & 1) ? ((w[e >> 1] & 0xffffu) | (b << 16)) : ((w[e >> 1] & 0xffff0000u) | b);
}
template <> struct Unit<__half> {
  static constexpr int E = 16;
  __device__ static float at(const uint32_t (&w)[8], int e) {
    float f;
    const unsigned short h = (unsigned short)(w[e >> 1] >> (16 * (e & 1)));
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return f;
  }
  __device__ static void put(uint32_t (&w)[8], int e, __half v) { put16(w, e, __half_as_ushort(v)); }
};
template <> struct Unit<__nv_bfloat16> {
  static constexpr int E = 16;
  __device__ static float at(const uint32_t (&w)[8], int e) {
    return __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
  }
  __device__ static void put(uint32_t (&w)[8], int e, __nv_bfloat16 v) { put16(w, e, __bfloat16_as_ushort(v)); }
};

__device__ __forceinline__ void load_unit(const unsigned char* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// NaN-propagating maximum of a unit (16-bit values: a packed-pair tree, two
// conversions at the end).
template <typename TIn>
__device__ __forceinline__ float unit_max(const uint32_t (&w)[8]) {
  using U = Unit<TIn>;
  if constexpr (U::E == 8) {
    const float a = max3_nan(U::at(w, 0), U::at(w, 1), U::at(w, 2));
    const float b = max3_nan(U::at(w, 3), U::at(w, 4), U::at(w, 5));
    return max3_nan(a, b, max_nan(U::at(w, 6), U::at(w, 7)));
  } else {
    auto mx2 = [](uint32_t x, uint32_t y) {
      uint32_t r;
      if constexpr (sizeof(TIn) == 2 && std::is_same<TIn, __half>::value)
        asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
      else
        asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
      return r;
    };
    const uint32_t p = mx2(mx2(mx2(w[0], w[1]), mx2(w[2], w[3])), mx2(mx2(w[4], w[5]), mx2(w[6], w[7])));
    const uint32_t q[8] = {p, 0, 0, 0, 0, 0, 0, 0};
    return max_nan(U::at(q, 0), U::at(q, 1));
  }
}

// Seen bits of elements e0 .. e0+E-1 (indices outside [0, V) give 0).
__device__ __forceinline__ uint32_t unit_bits(const uint32_t* bm, int64_t e0, int E, int64_t V) {
  if (e0 >= 0 && (int)(e0 & 31) + E <= 32 && e0 + E <= V)
    return (bm[e0 >> 5] >> (e0 & 31)) & (E == 32 ? ~0u : ((1u << E) - 1u));
  uint32_t r = 0;
  for (int e = 0; e < E; ++e) {
    const int64_t i = e0 + e;
    if (i >= 0 && i < V && ((bm[i >> 5] >> (i & 31)) & 1u)) r |= 1u << e;
  }
  return r;
}

// The bound from the histogram (one warp): the highest bin b with at least kk
// counted values in bins >= b gives key base + (b << shift).  Returns the lowered
// bound in the penalised domain, or -inf.  Lane l reads bins 8l .. 8l+7.
__device__ __forceinline__ float hist_bound(const unsigned int* bins, uint32_t base_key, int shift, int kk,
                                            float T) {
  const int lane = threadIdx.x & 31;
  // Volatile loads: other warps are still counting.
  uint32_t c[8];
  asm volatile("ld.volatile.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
               : "r"(smem_u32(bins + 8 * lane)));
  asm volatile("ld.volatile.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(c[4]), "=r"(c[5]), "=r"(c[6]), "=r"(c[7])
               : "r"(smem_u32(bins + 8 * lane + 4)));
  uint32_t s = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) s += c[q];
  uint32_t incl = s;  // count in bins of lanes >= lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += t;
  }
  int best = -1;
  uint32_t above = incl - s;
#pragma unroll
  for (int q = 7; q >= 0; --q) {
    above += c[q];
    if (best < 0 && above >= (uint32_t)kk) best = lane * 8 + q;
  }
  const unsigned m = __ballot_sync(0xffffffffu, best >= 0);
  if (!m) return Elem<float>::neg_inf();
  best = __shfl_sync(0xffffffffu, best, 31 - __clz(m));
  return lower_tau(key_to_float(base_key + ((uint32_t)best << shift)), T);
}

// One unit of a row by element loads, -inf outside the row: the partial units at
// a row's ends (out of line, so the batch loop keeps only the plain load).
struct UnitVals {
  uint4 a, b;
};

template <typename TIn>
__device__ __noinline__ UnitVals guarded_unit(const TIn* rowp, int u, int off_e, int nunits, int64_t V) {
  using U = Unit<TIn>;
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < U::E; ++e) {
    const int64_t i = (int64_t)u * U::E + e - off_e;
    U::put(w, e, (u < nunits && i >= 0 && i < V) ? rowp[i] : Elem<TIn>::neg_inf());
  }
  UnitVals r;
  r.a = make_uint4(w[0], w[1], w[2], w[3]);
  r.b = make_uint4(w[4], w[5], w[6], w[7]);
  return r;
}

// What a warp's queue drain needs besides the shared layout.
struct DrainCtx {
  float tau0, rp, T;
  int off_e, kk, bin_shift;
  uint32_t base_key;
};

template <int NT>
__device__ __forceinline__ float shared_tau(const StreamShared<NT>& sh, float tau0) {
  const float t = key_to_float(*reinterpret_cast<const volatile unsigned int*>(&sh.tau_key));
  return fmaxf(fmaxf(tau0, t), -3.402823466e38f);  // excludes -inf
}

// Drains the calling warp's queue of qn hit units, one unit per lane: each element
// whose penalised score reaches the current bound is appended to the warp's
// candidate list (count cnt, ballot-aggregated) and counted in the histogram; a
// list grown by RW entries since `last` recomputes the bound.  Returns {cnt, last}.
template <typename TIn, int NT>
__device__ __noinline__ int2 drain_queue(StreamShared<NT>* shp, const uint32_t* bits, int qn, int cnt, int last,
                                         DrainCtx c) {
  using U = Unit<TIn>;
  constexpr int E = U::E;
  constexpr int CAPW = CAP / (NT / 32);
  constexpr unsigned FULL = 0xffffffffu;
  StreamShared<NT>& sh = *shp;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lt_mask = (1u << lane) - 1u;
  float* wval = sh.cval() + warp * CAPW;
  int* widx = sh.cidx() + warp * CAPW;
  __syncwarp();  // the queue's stores are visible to the warp
  const float tc = shared_tau(sh, c.tau0);
  const bool have = lane < qn;
  uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int u = 0;
  if (have) {
    const uint4 p = sh.qdata(warp)[2 * lane], q = sh.qdata(warp)[2 * lane + 1];
    w[0] = p.x; w[1] = p.y; w[2] = p.z; w[3] = p.w;
    w[4] = q.x; w[5] = q.y; w[6] = q.z; w[7] = q.w;
    u = sh.qunit(warp)[lane];
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float x = U::at(w, e);
    bool pass = have && x >= tc;
    if (!__any_sync(FULL, pass)) continue;
    const int i = u * E + e - c.off_e;  // inside the row when pass: outside elements are -inf
    if (pass && ((bits[i >> 5] >> (i & 31)) & 1u)) {
      x = penalize(x, c.rp);
      pass = x >= tc;
    }
    const unsigned bal = __ballot_sync(FULL, pass);
    if (pass) {
      const int pos = cnt + __popc(bal & lt_mask);
      if (pos < CAPW) {
        wval[pos] = x;
        widx[pos] = i;
      }
      const uint32_t k = ord_key(x);
      if (k >= c.base_key)
        atomicAdd(&sh.bins[min((uint32_t)(SBINS - 1), (k - c.base_key) >> c.bin_shift)], 1u);
    }
    cnt += __popc(bal);
  }
  __syncwarp();  // the queue may be refilled
  if (cnt >= last + RW) {
    last = cnt;
    const float tb = hist_bound(sh.bins, c.base_key, c.bin_shift, c.kk, c.T);
    if (lane == 0 && tb > Elem<float>::neg_inf()) atomicMax(&sh.tau_key, ord_key(tb));
  }
  return make_int2(cnt, last);
}

// The history forms the bulk copy does not take (ids that are unaligned or too
// many for the staging region, the packed bitmap, the bool mask).
template <int NT>
__device__ __forceinline__ int mark_other(const RowArgs& a, int64_t row, int64_t V, uint32_t* bits) {
  const int tid = threadIdx.x;
  const int nw = (int)((V + 31) >> 5);
  int err = 0;
  if (a.hist_kind == HIST_IDS32 || a.hist_kind == HIST_IDS64) {
    const int64_t L = hist_length(a, row);
    for (int64_t j = tid; j < L; j += NT) {
      const int64_t x = hist_id(a, row, j);
      if ((uint64_t)x >= (uint64_t)V) {
        err |= 1 << ST_HISTORY;
      } else {
        const uint32_t b = 1u << (x & 31);
        if (!(bits[x >> 5] & b)) atomicOr(&bits[x >> 5], b);
      }
    }
  } else if (a.hist_kind == HIST_BITS32) {
    const uint32_t* hb = reinterpret_cast<const uint32_t*>(a.hist) + row * a.hist_stride;
    for (int w = tid; w < nw; w += NT) {
      uint32_t v = hb[w];
      if (w == nw - 1 && (V & 31)) v &= (1u << (V & 31)) - 1u;
      bits[w] = v;
    }
  } else if (a.hist_kind == HIST_MASK8) {
    for (int64_t i = tid; i < V; i += NT)
      if (seen_global(a, row, i)) atomicOr(&bits[i >> 5], 1u << (i & 31));
  }
  return err;
}

// Resident CTAs per SM the register budget is sized for: 7 x 128 threads (1036
// rows at once on 148 SMs), 3 x 256, 2 x 512.
template <int NT>
constexpr int min_blocks() {
  return NT == 128 ? 7 : NT == 256 ? 3 : 2;
}

template <typename TIn, int NT>
__global__ void __launch_bounds__(NT, min_blocks<NT>()) stream_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  using Sh = StreamShared<NT>;
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);
  BlockScratch<NT>& bs = sh.bs;
  uint32_t* bits = reinterpret_cast<uint32_t*>(smem_raw + static_bytes(NT));
  using U = Unit<TIn>;
  constexpr int E = U::E;
  constexpr int ES = Elem<TIn>::kSize;
  constexpr int NWARPS = NT / 32;
  constexpr int CAPW = CAP / NWARPS;  // candidates per warp list
  constexpr int BATCH = NT * BU;      // units per CTA batch
  static_assert(sizeof(SmallFin) <= NWARPS * QCAP * 32, "the small finish's state lies over the hit queues");
  constexpr unsigned FULL = 0xffffffffu;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float NEG = Elem<float>::neg_inf();
  const float PINF = __int_as_float(0x7f800000);
  const int64_t V = a.vocab;
  const int nw = (int)((V + 31) >> 5);
  const float rp = a.rep_penalty, T = a.temperature;
  const int kk = a.kk;
  const int64_t row = blockIdx.x;
  const unsigned lt_mask = (1u << lane) - 1u;

  // Row geometry: 32-byte units from the row start rounded down.
  const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
  const uintptr_t gs = reinterpret_cast<uintptr_t>(rowp);
  const uintptr_t ge = gs + (uintptr_t)V * ES;
  const uintptr_t b32 = gs & ~uintptr_t(UB - 1);
  const unsigned char* base = reinterpret_cast<const unsigned char*>(b32);
  const int off_e = (int)((gs - b32) / ES);
  const int nunits = (int)((ge - b32 + UB - 1) / UB);
  const int u_lo = gs == b32 ? 0 : 1;          // first unit inside the row
  const int u_hi = (int)((ge - b32) / UB);     // units [u_lo, u_hi) lie inside
  const int nb = (nunits + BATCH - 1) / BATCH;

  // Loads of batch b: whole batches inside the row take the 256-bit load; the
  // partial ones at the row's ends go through guarded_unit.
  const int bf0 = u_lo, bf1 = u_hi / BATCH;  // batches [bf0, bf1) lie inside the row
  auto load_batch = [&](uint32_t (&w)[BU][8], int b) {
    const int u = b * BATCH + tid;
    if ((b >= bf0 && b < bf1) || (u >= u_lo && u < u_hi)) {
      load_unit(base + (size_t)u * UB, w[0]);
    } else {
      const UnitVals r = guarded_unit<TIn>(rowp, u, off_e, nunits, V);
      w[0][0] = r.a.x; w[0][1] = r.a.y; w[0][2] = r.a.z; w[0][3] = r.a.w;
      w[0][4] = r.b.x; w[0][5] = r.b.y; w[0][6] = r.b.z; w[0][7] = r.b.w;
    }
  };

  // 0. the history ids by one bulk copy into the staging region when they fit it
  //    (larger or unaligned histories and the other history forms by plain loads).
  //    The first logits are loaded once the bitmap is built: loads outstanding
  //    during the bitmap build slow its shared-memory work.
  const bool ids_kind = a.hist_kind == HIST_IDS32 || a.hist_kind == HIST_IDS64;
  const int idb = a.hist_kind == HIST_IDS64 ? 8 : 4;
  const int64_t L = ids_kind ? hist_length(a, row) : 0;
  const unsigned char* hrow =
      ids_kind ? reinterpret_cast<const unsigned char*>(a.hist) + (size_t)row * a.hist_stride * idb : nullptr;
  const bool stage_ids = ids_kind && (reinterpret_cast<uintptr_t>(hrow) & 15) == 0 && L * idb <= kIdStage;
  const uint32_t tma_bytes = stage_ids ? (uint32_t)((L * idb) & ~int64_t(15)) : 0u;
  if (tid == 0) {
    mbar_init(&sh.idbar, 1);
    fence_proxy_async_smem();  // the initialised barrier is visible to the bulk copy
    if (tma_bytes) {
      // The test hook expects 16 bytes the copy never brings: the wait runs out.
      mbar_expect_tx(&sh.idbar, tma_bytes + (a.wait_test ? 16u : 0u));
      bulk_g2s(sh.stage, hrow, tma_bytes, &sh.idbar);
    }
  }
  uint32_t w0[1][8], w1[1][8], w2[1][8], w3[1][8];

  // 1. seen bitmap.
  {
    const int nz = (nw + 4 + 3) >> 2;  // 16-byte words, within bitmap_bytes(V)
    for (int q = tid; q < nz; q += NT) reinterpret_cast<uint4*>(bits)[q] = make_uint4(0, 0, 0, 0);
    for (int q = tid; q < SBINS / 4; q += NT) reinterpret_cast<uint4*>(sh.bins)[q] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
      sh.err = 0;
      sh.rmax_key = 0;
      sh.tau_key = ord_key(NEG);
    }
  }
  __syncthreads();
  {
    int e = 0;
    if (stage_ids) {
      // The ids past the last whole 16 bytes (fewer than four) by plain loads.
      const int64_t done = tma_bytes / idb;
      if (tid < L - done) {
        const int64_t x = hist_id(a, row, done + tid);
        if ((uint64_t)x >= (uint64_t)V) e |= 1 << ST_HISTORY;
        else atomicOr(&bits[x >> 5], 1u << (x & 31));
      }
      if (tma_bytes) {
        const uint64_t limit = a.wait_test ? 2000000ull : 1000000000ull;
        if (!__all_sync(FULL, mbar_wait(&sh.idbar, 0, limit))) {  // warp-uniform, for the reductions below
          e |= 1 << ST_TIMEOUT;
          (void)mbar_wait(&sh.idbar, 0, limit);  // let a late copy land before the region is reused
        } else {
          const uint4* st = reinterpret_cast<const uint4*>(sh.stage);
          const int nvec = (int)(tma_bytes >> 4);
          const uint32_t uV = (uint32_t)V;
          auto mark32 = [&](uint32_t x) {
            if (x >= uV) {
              e |= 1 << ST_HISTORY;
            } else {
              const uint32_t bm = 1u << (x & 31);
              uint32_t* wd = &bits[x >> 5];
              if (!(*wd & bm)) atomicOr(wd, bm);
            }
          };
          if (idb == 4) {
            for (int q = tid; q < nvec; q += NT) {
              const uint4 t = st[q];
              mark32(t.x);
              mark32(t.y);
              mark32(t.z);
              mark32(t.w);
            }
          } else {
            for (int q = tid; q < nvec; q += NT) {
              const uint4 t = st[q];
              mark32(t.y ? ~0u : t.x);
              mark32(t.w ? ~0u : t.z);
            }
          }
        }
      }
    } else {
      e = mark_other<NT>(a, row, V, bits);
    }
    if (e) atomicOr(&sh.err, e);
  }
  __syncthreads();

  // 2. the first bound: each thread's maximum over the unseen elements of the
  //    first RING batches; the smallest of the warps' ceil(kk / warps)-th largest
  //    maxima (at least kk elements of the row reach it).
  load_batch(w0, 0);
  load_batch(w1, 1);
  load_batch(w2, 2);
  load_batch(w3, 3);
  float boot;
  {
    float g = NEG;
    auto boot_unit = [&](const uint32_t (&w)[1][8], int u) {
      const int64_t e0 = (int64_t)u * E - off_e;
      const uint32_t sb = off_e == 0 && u < u_hi ? (bits[e0 >> 5] >> (e0 & 31)) & ((1u << E) - 1u)
                                                 : unit_bits(bits, e0, E, V);
      if (!sb) {
        g = max_nan(g, unit_max<TIn>(w[0]));
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (!((sb >> e) & 1u)) g = fmaxf(g, U::at(w[0], e));
      }
    };
    boot_unit(w0, tid);
    boot_unit(w1, BATCH + tid);
    boot_unit(w2, 2 * BATCH + tid);
    boot_unit(w3, 3 * BATCH + tid);
    if (g != g) g = NEG;  // NaN rows fail with ST_NAN; keep the ranks well defined
    int rank = 0;
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const float o = __shfl_sync(FULL, g, q);
      rank += (o > g) || (o == g && q < lane);
    }
    sh.wsort[warp][rank] = g;
    __syncthreads();
    // Every warp holds jw values >= its jw-th largest: NWARPS * jw >= kk values
    // reach the smallest of those, a valid first bound.
    const int jw = (kk + NWARPS - 1) / NWARPS;
    float b = sh.wsort[0][jw - 1];
#pragma unroll
    for (int ow = 1; ow < NWARPS; ++ow) b = fminf(b, sh.wsort[ow][jw - 1]);
    boot = b;
  }
  float hi_boot = sh.wsort[0][0];
#pragma unroll
  for (int ow = 1; ow < NWARPS; ++ow) hi_boot = fmaxf(hi_boot, sh.wsort[ow][0]);
  const uint32_t base_key = ord_key(boot);
  int bin_shift = 0;
  {
    const uint32_t span = ord_key(hi_boot) > base_key ? ord_key(hi_boot) - base_key : 0u;
    while ((span >> bin_shift) >= (uint32_t)SBINS) ++bin_shift;
  }
  const float tau0 = lower_tau(boot, T);

  // 3. batches.  A unit whose maximum reaches the bound is queued (its 32 bytes
  //    and unit number) in the warp's queue; a full queue is drained, one unit per
  //    lane.  The bound is read from shared memory once per ring turn and after
  //    each drain.
  float rmx = NEG;  // NaN-propagating maximum of this thread's raw scores
  int cnt = 0;      // this warp's candidates (warp-uniform)
  int last = 0;     // cnt at the warp's last bound recomputation
  int qn = 0;       // queued units (warp-uniform)
  const DrainCtx dc = {tau0, rp, T, off_e, kk, bin_shift, base_key};
  float tc = shared_tau(sh, tau0);
  auto process = [&](const uint32_t (&w)[BU][8], int b) {
    const float um = unit_max<TIn>(w[0]);
    rmx = max_nan(rmx, um);
    const bool hit = um >= tc;
    const unsigned bal = __ballot_sync(FULL, hit);
    if (bal) {
      const int n = __popc(bal);
      if (qn + n > QCAP) {
        const int2 r = drain_queue<TIn, NT>(&sh, bits, qn, cnt, last, dc);
        cnt = r.x;
        last = r.y;
        qn = 0;
        tc = shared_tau(sh, tau0);
      }
      if (hit) {
        const int pos = qn + __popc(bal & lt_mask);
        sh.qdata(warp)[2 * pos] = make_uint4(w[0][0], w[0][1], w[0][2], w[0][3]);
        sh.qdata(warp)[2 * pos + 1] = make_uint4(w[0][4], w[0][5], w[0][6], w[0][7]);
        sh.qunit(warp)[pos] = b * BATCH + tid;
      }
      qn += n;
    }
  };
  for (int b = 0; b < nb; b += RING) {
    process(w0, b);
    if (b + RING < nb) load_batch(w0, b + RING);
    if (b + 1 < nb) {
      process(w1, b + 1);
      if (b + 1 + RING < nb) load_batch(w1, b + 1 + RING);
    }
    if (b + 2 < nb) {
      process(w2, b + 2);
      if (b + 2 + RING < nb) load_batch(w2, b + 2 + RING);
    }
    if (b + 3 < nb) {
      process(w3, b + 3);
      if (b + 3 + RING < nb) load_batch(w3, b + 3 + RING);
    }
    tc = shared_tau(sh, tau0);
  }
  if (qn) {
    const int2 r = drain_queue<TIn, NT>(&sh, bits, qn, cnt, last, dc);
    cnt = r.x;
  }

  // 4. finish the row.
  if (rmx != rmx) atomicOr(&sh.err, 1 << ST_NAN);
  else if (rmx == PINF) atomicOr(&sh.err, 1 << ST_POSINF);
  rmx = warp_max_nan(rmx);
  if (lane == 0) {
    if (rmx == rmx) atomicMax(&sh.rmax_key, ord_key(rmx));
    sh.wcount[warp] = cnt;
  }
  if (tid == 0) {
    bs.flag = 0;
    sh.mkey = 0;
  }
  __syncthreads();
  // The final bound from the complete bins (every warp computes the same value).
  const float tfin = fmaxf(shared_tau(sh, tau0), hist_bound(sh.bins, base_key, bin_shift, kk, T));
  const float uu = a.uniforms[row];
  bool overflow = false;
#pragma unroll
  for (int ow = 0; ow < NWARPS; ++ow) overflow |= sh.wcount[ow] > CAPW;
  int status = sh.err ? first_err(sh.err) : ST_OK;
  bool general = status == ST_OK && a.force_slow;
  float* fv = sh.fv();
  int* fi = sh.fi();
  // Finish scratch in the candidate lists (consumed by then).
  float* sval = sh.cval();
  int* sidx = reinterpret_cast<int*>(sh.cval() + SFIN);
  uint64_t* Wb = reinterpret_cast<uint64_t*>(sh.cval() + 2 * SFIN);
  uint64_t* Pb = reinterpret_cast<uint64_t*>(sh.cidx());
  int* kidx = sh.cidx() + 2 * SFIN;
  float* kval = reinterpret_cast<float*>(sh.cidx());
  int m = 0;
  if (status == ST_OK && !general) {
    // The candidates whose penalised score reaches the final bound, tempered.
    if (overflow) {
      // A list overflowed: the row is read again (from L2 or HBM).
      int bad = 0;
      auto take = [&](int i, float x) {
        const float tx = temper(x, T);
        bad |= tx == PINF;
        const int at = atomicAdd(&bs.flag, 1);
        if (at < SFIN) {
          fv[at] = tx;
          fi[at] = i;
        }
      };
      for (int64_t i = tid; i < V; i += NT) {
        float x = Elem<TIn>::load(rowp + i);
        if (x >= tfin) {
          if ((bits[i >> 5] >> (i & 31)) & 1u) x = penalize(x, rp);
          if (x >= tfin) take((int)i, x);
        }
      }
      if (bad) atomicOr(&sh.err, 1 << ST_POSINF);
      __syncthreads();
      m = bs.flag;
      if (sh.err) status = first_err(sh.err);
      __syncthreads();
    } else {
      // Each warp compacts its own list: counts first, then every warp writes its
      // entries after the lists before it (the finish input is ordered by warp
      // list, then by position in the list).
      const int n = sh.wcount[warp];
      const float* lv = sh.cval() + warp * CAPW;
      const int* li = sh.cidx() + warp * CAPW;
      int c = 0;
      bool bad = false;
      float mx = NEG;
      for (int b0 = 0; b0 < n; b0 += 32) {
        const float x = b0 + lane < n ? lv[b0 + lane] : NEG;
        const bool pass = x >= tfin;
        const float tx = pass ? temper(x, T) : NEG;
        bad |= tx == PINF;
        mx = fmaxf(mx, tx);
        c += __popc(__ballot_sync(FULL, pass));
      }
      mx = warp_max_nan(mx);
      bad = __any_sync(FULL, bad);
      if (lane == 0) {
        sh.ccount[warp] = c;
        if (bad) atomicOr(&sh.err, 1 << ST_POSINF);
        if (mx > NEG) atomicMax(&sh.mkey, ord_key(mx));
      }
      __syncthreads();
      int off = 0;
#pragma unroll
      for (int ow = 0; ow < NWARPS; ++ow) {
        if (ow < warp) off += sh.ccount[ow];
        m += sh.ccount[ow];
      }
      for (int b0 = 0; b0 < n; b0 += 32) {
        const float x = b0 + lane < n ? lv[b0 + lane] : NEG;
        const bool pass = x >= tfin;
        const unsigned bal = __ballot_sync(FULL, pass);
        const int pos = off + __popc(bal & lt_mask);
        if (pass && pos < SFIN) {
          fv[pos] = temper(x, T);
          fi[pos] = li[b0 + lane];
        }
        off += __popc(bal);
      }
      if (sh.err) status = first_err(sh.err);
      __syncthreads();
    }
    if (m > SFIN) general = status == ST_OK;
  }
  if (general && temper(key_to_float(sh.rmax_key), T) == PINF) {
    // A score may reach +inf only through the temperature: check every element.
    int inf = 0;
    for (int64_t i = tid; i < V; i += NT) {
      float x = Elem<TIn>::load(rowp + i);
      if ((bits[i >> 5] >> (i & 31)) & 1u) x = penalize(x, rp);
      inf |= temper(x, T) == PINF;
    }
    if (__syncthreads_or(inf)) {
      status = ST_POSINF;
      general = false;
    }
  }
  if (status == ST_OK && !general && m == 0) status = ST_ALLNEGINF;
  const bool dense = a.out_dense && a.dense_mode != DENSE_NONE;
  if (status == ST_OK && !general && m <= 64 && !dense && !overflow) {
    // Common case: the block finishes the row, two threads per candidate; its
    // scratch is the hit queues (dead by now) and the kept list goes over the
    // finish input.
    int64_t tok = -1;
    const Kept kp = finish_small<NT>(a, fv, fi, m, key_to_float(sh.mkey), uu, &tok, fi, fv,
                                     *reinterpret_cast<SmallFin*>(sh.qdata(0)));
    const float Sf = fix_to_float(kp.tot);
    for (int j = tid; j < kp.n && j < a.out_cap; j += NT) {
      if (a.out_idx) a.out_idx[row * a.out_cap + j] = fi[j];
      if (a.out_prob) a.out_prob[row * a.out_cap + j] = __fdiv_rn(sv_exp(__fsub_rn(fv[j], kp.M)), Sf);
      if (a.out_score) a.out_score[row * a.out_cap + j] = fv[j];
    }
    if (tid == 0) {
      a.out_token[row] = tok;
      if (a.out_count) a.out_count[row] = kp.n;
      if (a.out_status) a.out_status[row] = ST_OK;
      if (a.seen_bits && tok >= 0) atomicOr(&a.seen_bits[row * a.seen_bits_stride + (tok >> 5)], 1u << (tok & 31));
    }
    return;
  }
  Kept kept = {0, 0.0f, 0};
  int64_t token = -1;
  if (dense && status == ST_OK && !general) {
    const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
    for (int64_t i = tid; i < V; i += NT) a.out_dense[row * a.dense_stride + i] = dv;
    __syncthreads();
  }
  if (status == ST_OK && !general) {
    if (m <= 64) {
      if (warp == 0) {
        kept = warp_finish<2>(a, fv, fi, m, uu, &token, kidx, kval);
        if (lane == 0) {
          bs.flag2 = kept.n;
          bs.fval = kept.M;
          bs.u64a = kept.tot;
        }
      }
      __syncthreads();
      kept.n = bs.flag2;
      kept.M = bs.fval;
      kept.tot = bs.u64a;
    } else {
      kept = leader_fast<NT>(a, bs, fv, fi, m, sval, sidx, Wb, Pb, kidx, kval);
      token = draw_kept<NT>(bs, kidx, kval, kept, uu, reinterpret_cast<uint64_t*>(sh.cval()));
    }
    const float Sf = fix_to_float(kept.tot);
    for (int j = tid; j < kept.n; j += NT) {
      const float p = __fdiv_rn(sv_exp(__fsub_rn(kval[j], kept.M)), Sf);
      if (j < a.out_cap) {
        if (a.out_idx) a.out_idx[row * a.out_cap + j] = kidx[j];
        if (a.out_prob) a.out_prob[row * a.out_cap + j] = p;
        if (a.out_score) a.out_score[row * a.out_cap + j] = kval[j];
      }
      if (dense) a.out_dense[row * a.dense_stride + kidx[j]] = a.dense_mode == DENSE_SCORES ? kval[j] : p;
    }
  } else if (general) {
    auto seen = [&](int64_t i) -> bool { return (bits[i >> 5] >> (i & 31)) & 1u; };
    auto emit = [&](int pos, int idx, float val, float Sf, float M) {
      if (pos < a.out_cap) {
        if (a.out_idx) a.out_idx[row * a.out_cap + pos] = idx;
        if (a.out_prob) a.out_prob[row * a.out_cap + pos] = __fdiv_rn(sv_exp(__fsub_rn(val, M)), Sf);
        if (a.out_score) a.out_score[row * a.out_cap + pos] = val;
      }
    };
    kept = leader_slow<NT, TIn, MODE_SAMPLE>(a, bs, reinterpret_cast<unsigned char*>(sh.cval()), row, 0.0f, 0.0f, uu,
                                             &token, seen, emit);
  } else if (dense) {
    const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
    for (int64_t i = tid; i < V; i += NT) a.out_dense[row * a.dense_stride + i] = dv;
  }
  if (tid == 0) {
    a.out_token[row] = status == ST_OK ? token : -1;
    if (a.out_count) a.out_count[row] = kept.n;
    if (a.out_status) a.out_status[row] = status;
    if (status == ST_OK && a.seen_bits && token >= 0)
      atomicOr(&a.seen_bits[row * a.seen_bits_stride + (token >> 5)], 1u << (token & 31));
  }
}

// Threads per row: enough warps in flight over the whole GPU (about 32 per SM)
// whatever the row count.
int threads_for(int rows, int sms) {
  if (rows >= sms * 6) return 128;
  if (rows >= sms) return 256;  // 256 rows (config 5): 256 threads beat 512 by ~1 us
  return 512;
}

template <typename TIn, int NT>
cudaError_t launch_nt(const RowArgs& a, size_t smem, cudaStream_t stream, int dev) {
  auto kern = stream_kernel<TIn, NT>;
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_limit_stream());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  kern<<<a.rows, NT, smem + static_bytes(NT), stream>>>(a);
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_stream_t(const RowArgs& a, size_t smem, cudaStream_t stream) {
  static int sms[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!sms[dev]) {
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  switch (threads_for(a.rows, sms[dev])) {
    case 128: return launch_nt<TIn, 128>(a, smem, stream, dev);
    case 256: return launch_nt<TIn, 256>(a, smem, stream, dev);
    default: return launch_nt<TIn, 512>(a, smem, stream, dev);
  }
}

}  // namespace

// Shared memory of the batched kernel beyond its largest static layout (the row's
// seen bitmap), or 0 when the row's bitmap would leave too little room for
// several CTAs per SM (the cluster kernel then takes the rows).
size_t stream_smem_bytes(int64_t vocab) {
  const size_t s = bitmap_bytes(vocab);
  return s + static_bytes(512) <= 96 * 1024 ? s : 0;
}

cudaError_t launch_stream(const RowArgs& a, size_t smem, cudaStream_t stream) {
  if (a.dtype == DT_F32) return launch_stream_t<float>(a, smem, stream);
  if (a.dtype == DT_F16) return launch_stream_t<__half>(a, smem, stream);
  return launch_stream_t<__nv_bfloat16>(a, smem, stream);
}

}  // namespace sv
