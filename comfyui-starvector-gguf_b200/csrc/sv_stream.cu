// sv_stream.cu -- the streaming row kernel (sm_100a): many independent rows.
//
// Persistent CTAs work through their rows one at a time.  A row's
// logits (and, ahead of them, its history ids) stream through a per-CTA ring of
// shared-memory slots filled by TMA bulk copies (cp.async.bulk, one mbarrier per
// slot); the ring runs ahead across row boundaries, so HBM keeps streaming while
// the CTA computes or finishes a row.
//
// Per row (runtime_shared.py:200-202):
//   1. the row's seen bitmap in shared memory, from the history;
//   2. per chunk, one pass over 16-byte units: the unit maximum of the raw scores
//      is tested against the current lower bound tau of the row's k-th largest
//      penalised score, and the units that reach it are kept (their 16 bytes and
//      seen bits).  The units also feed 128 lane-pair group values, a unit with a
//      seen token through a lower bound of its penalised maximum (each group value
//      is at or below a distinct element of its group, so the k-th largest group
//      value bounds the row's k-th largest from below).  In the first chunk the
//      exact k-th largest of the chunk's group values gives the first bound;
//      later group values go into a 256-bin histogram over ordered float keys,
//      whose highest bin edge with at least k values at or above it is a
//      tightening bound;
//   3. finish: the kept units' elements whose penalised score (:172-173) reaches
//      the final bound are the candidates, tempered (:178-179); then the exact
//      k-th largest with ties (:180-181), top-p over the ascending (value, index)
//      order with exact fixed-point mass (:182-186) and the draw from the row's
//      uniform, by one warp for up to 64 candidates.  A row with too many (huge tie
//      groups) takes the general path over the whole row.
// Status: a NaN anywhere in the row, else a +inf tempered score, else no finite
// score.  No inter-CTA communication and no scratch memory in global memory.
#include <cuda_runtime.h>

#include "sv_block.cuh"
#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

namespace {

// Resident CTAs per SM: 3 (256 threads, a 3-slot ring each) or 1 (512 threads, a
// 12-slot ring).
#ifndef SV_STREAM_CTAS_PER_SM
#define SV_STREAM_CTAS_PER_SM 3
#endif
constexpr int kCtasPerSm = SV_STREAM_CTAS_PER_SM;
constexpr int SNT = kCtasPerSm == 1 ? 512 : 256;  // threads per CTA
constexpr int SWARPS = SNT / 32;
constexpr int SBUF = kCtasPerSm == 1 ? 12 : 3;  // ring slots
constexpr size_t kSmemCap = kCtasPerSm == 1 ? 227 * 1024 : 74 * 1024;  // per CTA
constexpr int SCHUNK = 16 * 1024;       // bytes per slot / chunk
constexpr int SCU = SCHUNK / 16;        // 16-byte units per chunk
constexpr int UPT = SCU / SNT;          // units per thread per chunk
constexpr int SBINS = 256;              // bound histogram bins
constexpr int UCAP = 704;               // hit units per row (their 16 bytes are kept)
constexpr int SFIN = 256;               // candidates the fast finish handles after pruning
constexpr int kBoundWarp = SWARPS - 1;  // computes the histogram bound after each chunk
constexpr int kIssuer = 32;             // issues the bulk copies (warp 1: warp 0 may be finishing a row)
constexpr int NB = SNT - 32;            // threads of warps 1.. that build a row's seen bitmap

struct __align__(16) StreamShared {
  unsigned long long mbar[SBUF];
  BlockScratch<SNT> bs;
  __align__(16) unsigned int bins[SBINS];
  float gsort[SWARPS][16];  // first chunk: each warp's group values, descending
  float first_raw;          //              and their kk-th largest
  float te_pub;           // bound published by the bound warp, read after the next barrier
  unsigned int rmax_key;  // ordered key of the row's largest raw score
  int unit_n;
  int err;
  __align__(16) uint4 udata[UCAP];  // hit units' 16 bytes; after the prune: finish scratch
  int uidx[UCAP];                   // hit units: (unit << 8) | seen bits
  __align__(16) unsigned char work[16 * SFIN];  // finish arrays / general-path scratch
};

constexpr size_t kStaticBytes = (sizeof(StreamShared) + 127) & ~size_t(127);

__host__ __device__ inline size_t bitmap_bytes(int64_t V) {
  return (((size_t)V + 31) / 32 * 4 + 16 + 127) & ~size_t(127);
}

// Warps 1.. only (the row-start bitmap build, while warp 0 may still finish the
// previous row).
__device__ __forceinline__ void bar_builders() { asm volatile("bar.sync 1, %0;" ::"n"(NB) : "memory"); }

// Geometry of one row's window: 16-byte units from the row start rounded down.
struct RowGeom {
  const unsigned char* base16;  // first unit
  uintptr_t b_lo, b_hi;         // 16-byte-aligned interior [b_lo, b_hi)
  int off_e;                    // window position of element 0
  int nunits;
  int nch;                      // chunks
};

template <typename TIn>
__device__ __forceinline__ RowGeom row_geom(const RowArgs& a, int64_t row) {
  constexpr int ES = Elem<TIn>::kSize;
  const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
  const uintptr_t gs = reinterpret_cast<uintptr_t>(rowp);
  const uintptr_t ge = gs + (uintptr_t)a.vocab * ES;
  RowGeom g;
  const uintptr_t b16 = gs & ~uintptr_t(15);
  g.base16 = reinterpret_cast<const unsigned char*>(b16);
  g.off_e = (int)((gs - b16) / ES);
  g.nunits = (int)((ge - b16 + 15) / 16);
  g.nch = (g.nunits + SCU - 1) / SCU;
  g.b_lo = (gs + 15) & ~uintptr_t(15);
  g.b_hi = ge & ~uintptr_t(15);
  return g;
}

// Issue chunk c of the row described by g into `slot` (one thread).
__device__ __forceinline__ void issue_chunk(const RowGeom& g, int c, unsigned char* slot, void* bar) {
  const uintptr_t w0 = reinterpret_cast<uintptr_t>(g.base16) + (uintptr_t)c * SCHUNK;
  const uintptr_t w1 = reinterpret_cast<uintptr_t>(g.base16) + (uintptr_t)g.nunits * 16;
  const uintptr_t lo = w0 > g.b_lo ? w0 : g.b_lo;
  uintptr_t hi = w0 + SCHUNK < w1 ? w0 + SCHUNK : w1;
  if (hi > g.b_hi) hi = g.b_hi;
  if (hi > lo) {
    const uint32_t bytes = (uint32_t)(hi - lo);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(slot + (lo - w0), reinterpret_cast<const void*>(lo), bytes, bar);
  } else {
    mbar_arrive(bar);
  }
}

// Seen bits of elements e0 .. e0+E-1 (indices outside [0, V) give 0).
__device__ __forceinline__ uint32_t unit_bits(const uint32_t* bm, int64_t e0, int E, int64_t V) {
  if (e0 >= 0 && (int)(e0 & 31) + E <= 32) return (bm[e0 >> 5] >> (e0 & 31)) & ((1u << E) - 1u);
  uint32_t r = 0;
  for (int e = 0; e < E; ++e) {
    const int64_t i = e0 + e;
    if (i >= 0 && i < V && ((bm[i >> 5] >> (i & 31)) & 1u)) r |= 1u << e;
  }
  return r;
}

// The bound from the histogram (one warp): the highest bin b with at least kk group
// maxima in bins >= b gives key base + (b << shift).  Returns the lowered bound in
// the penalised domain, or -inf.  Lane l reads bins 8l .. 8l+7.
__device__ __forceinline__ float hist_bound(const unsigned int* bins, uint32_t base_key, int shift, int kk,
                                            float T) {
  const int lane = threadIdx.x & 31;
  const uint4 b0 = reinterpret_cast<const uint4*>(bins)[2 * lane];
  const uint4 b1 = reinterpret_cast<const uint4*>(bins)[2 * lane + 1];
  const uint32_t c[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
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
  // The highest lane with a qualifying bin holds the answer.
  const unsigned m = __ballot_sync(0xffffffffu, best >= 0);
  if (!m) return Elem<float>::neg_inf();
  best = __shfl_sync(0xffffffffu, best, 31 - __clz(m));
  return lower_tau(key_to_float(base_key + ((uint32_t)best << shift)), T);
}

// Marks history ids staged in shared memory (16-byte vectors of Id) in the bitmap
// (threads 32..); returns the ST_HISTORY error bit for ids outside [0, V).
template <typename Id>
__device__ __forceinline__ int mark_staged(const unsigned char* src, int64_t L, int64_t V, uint32_t* bits) {
  constexpr int PER = 16 / (int)sizeof(Id);
  int err = 0;
  for (int64_t q = threadIdx.x - 32; q * PER < L; q += NB) {
    Id id[PER];
    *reinterpret_cast<uint4*>(id) = reinterpret_cast<const uint4*>(src)[q];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      if (q * PER + t >= L) break;
      const int64_t x = (int64_t)id[t];
      if (x < 0 || x >= V) {
        err |= 1 << ST_HISTORY;
      } else {
        const uint32_t b = 1u << (x & 31);
        uint32_t* w = &bits[x >> 5];
        if (!(*w & b)) atomicOr(w, b);  // repeated ids mostly find their bit set
      }
    }
  }
  return err;
}

template <typename TIn>
__global__ void __launch_bounds__(SNT, kCtasPerSm) stream_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StreamShared& sh = *reinterpret_cast<StreamShared*>(smem_raw);
  BlockScratch<SNT>& bs = sh.bs;
  unsigned char* ring = smem_raw + kStaticBytes;
  uint32_t* bits = reinterpret_cast<uint32_t*>(ring + (size_t)SBUF * SCHUNK);
  constexpr int ES = Elem<TIn>::kSize;
  constexpr int EPU = 16 / ES;
  using IO = UnitIO<TIn>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float NEG = Elem<float>::neg_inf();
  const float PINF = __int_as_float(0x7f800000);
  const int64_t V = a.vocab;
  const int nw = (int)((V + 31) >> 5);
  const float rp = a.rep_penalty, T = a.temperature;
  const float rinv_lo = __frcp_rd(rp);  // <= 1/rp: x * rinv_lo rounded down <= x / rp rounded
  const int kk = a.kk;
  const int64_t first = blockIdx.x, step = gridDim.x;
  if (first >= a.rows) return;

  // History ids travel through the ring ahead of their row when they fit a slot.
  const bool ids_kind = a.hist_kind == HIST_IDS32 || a.hist_kind == HIST_IDS64;
  const int idb = a.hist_kind == HIST_IDS64 ? 8 : 4;
  const size_t hbytes = ids_kind ? (size_t)a.hist_cols * idb : 0;
  const bool stage_ids = ids_kind && hbytes > 0 && hbytes <= SCHUNK && hbytes % 16 == 0 &&
                         (reinterpret_cast<uintptr_t>(a.hist) % 16) == 0 && ((size_t)a.hist_stride * idb) % 16 == 0;

  // Issue cursor (thread 0 only): ic = -1 is the row's ids, then its chunks.
  int64_t irow = first;
  int ic = stage_ids ? -1 : 0;
  RowGeom ig = row_geom<TIn>(a, irow);
  int islot = 0;  // ring slot of the next issue
  if (tid == 0) {
    for (int s = 0; s < SBUF; ++s) mbar_init(&sh.mbar[s], 1);
    mbar_init_fence();
    sh.err = 0;
  }
  __syncthreads();
  auto issue_next = [&]() {  // thread kIssuer, after a barrier
    if (irow >= a.rows) return;
    fence_proxy_async_smem();
    const int s = islot;
    unsigned char* slot = ring + (size_t)s * SCHUNK;
    if (ic < 0) {
      mbar_expect_tx(&sh.mbar[s], (uint32_t)hbytes);
      bulk_g2s(slot, reinterpret_cast<const unsigned char*>(a.hist) + (size_t)irow * a.hist_stride * idb,
               (uint32_t)hbytes, &sh.mbar[s]);
    } else {
      issue_chunk(ig, ic, slot, &sh.mbar[s]);
    }
    if (++islot == SBUF) islot = 0;
    if (++ic == ig.nch) {
      ic = stage_ids ? -1 : 0;
      irow += step;
      if (irow < a.rows) ig = row_geom<TIn>(a, irow);
    }
  };
  if (tid == kIssuer)
    for (int s = 0; s < SBUF; ++s) issue_next();

  // Ring slot and mbarrier phase of the next slot to consume (all threads).
  int cslot = 0;
  uint32_t cphase = 0;
  auto consume_next = [&]() {
    if (++cslot == SBUF) {
      cslot = 0;
      cphase ^= 1u;
    }
  };

  for (int64_t row = first; row < a.rows; row += step) {
    const RowGeom g = row_geom<TIn>(a, row);
    const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
    const bool aligned = g.off_e == 0;
    // 1. seen bitmap of the row, by warps 1.. (warp 0 may still be finishing the
    //    previous row; it joins at the barrier before the chunks).
    if (warp > 0) {
      const int bt = tid - 32;
      {
        const int nz = (nw + 4 + 3) >> 2;  // 16-byte words, within bitmap_bytes(V)
        for (int w = bt; w < nz; w += NB) reinterpret_cast<uint4*>(bits)[w] = make_uint4(0, 0, 0, 0);
      }
      if (bt < SBINS / 4) reinterpret_cast<uint4*>(sh.bins)[bt] = make_uint4(0, 0, 0, 0);
      if (tid == kIssuer) {
        sh.unit_n = 0;
        sh.te_pub = NEG;
        sh.rmax_key = 0;
        sh.err = 0;
      }
      bar_builders();
      int local_err = 0;
      if (ids_kind) {
        const int64_t L = hist_length(a, row);
        if (stage_ids) {
          if (!mbar_wait(&sh.mbar[cslot], cphase)) local_err |= 1 << ST_TIMEOUT;
          const unsigned char* src = ring + (size_t)cslot * SCHUNK;
          local_err |= idb == 4 ? mark_staged<int32_t>(src, L, V, bits) : mark_staged<int64_t>(src, L, V, bits);
          bar_builders();  // the ids slot is consumed
          if (tid == kIssuer) issue_next();
        } else {
          for (int64_t j = bt; j < L; j += NB) {
            const int64_t x = hist_id(a, row, j);
            if (x < 0 || x >= V) {
              local_err |= 1 << ST_HISTORY;
            } else {
              const uint32_t b = 1u << (x & 31);
              if (!(bits[x >> 5] & b)) atomicOr(&bits[x >> 5], b);
            }
          }
        }
      } else if (a.hist_kind == HIST_BITS32) {
        const uint32_t* hb = reinterpret_cast<const uint32_t*>(a.hist) + row * a.hist_stride;
        for (int w = bt; w < nw; w += NB) {
          uint32_t v = hb[w];
          if (w == nw - 1 && (V & 31)) v &= (1u << (V & 31)) - 1u;
          bits[w] = v;
        }
      } else if (a.hist_kind == HIST_MASK8) {
        for (int64_t i = bt; i < V; i += NB)
          if (seen_global(a, row, i)) atomicOr(&bits[i >> 5], 1u << (i & 31));
      }
      if (local_err) atomicOr(&sh.err, local_err);
    }
    if (stage_ids) consume_next();  // every thread keeps the ring position
    __syncthreads();

    // 2. chunks.
    float te = NEG;         // current bound (penalised domain)
    float rmx = NEG;        // NaN-propagating maximum of this thread's raw scores
    uint32_t base_key = 0;  // histogram origin and bin width (identical in all threads)
    int bin_shift = 0;
    for (int c = 0; c < g.nch; ++c, consume_next()) {
      TIn* slot = reinterpret_cast<TIn*>(ring + (size_t)cslot * SCHUNK);
      if (!mbar_wait(&sh.mbar[cslot], cphase)) atomicOr(&sh.err, 1 << ST_TIMEOUT);
      const int u0 = c * SCU;
      const int un = min(SCU, g.nunits - u0);
      // Ragged units (outside the aligned interior) come from global memory, with
      // -inf outside the row; each unit belongs to one thread.
      if (!aligned || un < SCU || g.b_hi < reinterpret_cast<uintptr_t>(g.base16) + (uintptr_t)g.nunits * 16) {
        for (int k = tid; k < un; k += SNT) {
          const uintptr_t ua = reinterpret_cast<uintptr_t>(g.base16) + (uintptr_t)(u0 + k) * 16;
          if (ua < g.b_lo || ua >= g.b_hi) {
#pragma unroll
            for (int e = 0; e < EPU; ++e) {
              const int64_t ei = (int64_t)(u0 + k) * EPU + e - g.off_e;
              slot[k * EPU + e] = (ei >= 0 && ei < V) ? __ldg(rowp + ei) : Elem<TIn>::neg_inf();
            }
          }
        }
      }
      // Unit maxima, seen bits and this lane's group value.  A unit with a seen
      // token enters the group value through a lower bound of its penalised
      // maximum.  Full chunks
      // of aligned rows (the common case) take a path without bounds checks, their
      // units at a fixed bit offset in consecutive bitmap words.
      float umax[UPT];
      uint32_t sb[UPT];
      float gsrc = NEG;
      auto unit = [&](int j, const float (&v)[EPU], float m, uint32_t bitsj) {
        // At or below the unit's penalised maximum (the penalty is monotone and
        // never raises a score; its lower bounds are products rounded down, no
        // division): for a unit with a seen token, the penalty bound of its raw
        // maximum, or, when that maximum reaches the bound (only such values can
        // enter the histogram), the larger of its unseen elements' maximum and the
        // penalty bound of its largest seen element.
        float gv = m;
        if (bitsj) {
          gv = __fmul_rd(m, m < 0.0f ? rp : rinv_lo);
          if (m >= te) {
            float mu = NEG, ms = NEG;
#pragma unroll
            for (int e = 0; e < EPU; ++e) {
              if ((bitsj >> e) & 1u) ms = fmaxf(ms, v[e]);
              else mu = fmaxf(mu, v[e]);
            }
            gv = fmaxf(mu, __fmul_rd(ms, ms < 0.0f ? rp : rinv_lo));
          }
        }
        umax[j] = m;
        sb[j] = bitsj;
        rmx = max_nan(rmx, m);
        gsrc = fmaxf(gsrc, gv);  // fmaxf drops NaN; rmx reports it
      };
      if (aligned && un == SCU) {
        const int e0 = (u0 + tid) * EPU;
        const uint32_t* bw = bits + (e0 >> 5);
        const int shf = e0 & 31;
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          float v[EPU];
          IO::load(slot, tid + j * SNT, v);
          float m = v[0];
#pragma unroll
          for (int e = 1; e < EPU; ++e) m = max_nan(m, v[e]);
          unit(j, v, m, (bw[j * (SNT * EPU / 32)] >> shf) & ((1u << EPU) - 1u));
        }
      } else {
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          const int k = tid + j * SNT;
          float m = NEG;
          uint32_t b = 0;
          float v[EPU];
#pragma unroll
          for (int e = 0; e < EPU; ++e) v[e] = NEG;
          if (k < un) {
            b = aligned ? (bits[((u0 + k) * EPU) >> 5] >> (((u0 + k) * EPU) & 31)) & ((1u << EPU) - 1u)
                        : unit_bits(bits, (int64_t)(u0 + k) * EPU - g.off_e, EPU, V);
            IO::load(slot, k, v);
            m = v[0];
#pragma unroll
            for (int e = 1; e < EPU; ++e) m = max_nan(m, v[e]);
          }
          unit(j, v, m, b);
        }
      }
      const float gm = fmaxf(gsrc, __shfl_xor_sync(0xffffffffu, gsrc, 1));  // lane-pair group value
      if (c == 0) {
        // First bound: the exact kk-th largest of the chunk's 128 group values in
        // the order (value desc, warp, group).  Each warp sorts its 16 by rank; a
        // value's global rank adds its position in the other warps' lists (binary
        // search); the value of rank kk - 1 is the bound.
        const int pair = lane >> 1;
        int rank = 0;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float w = __shfl_sync(0xffffffffu, gm, 2 * q);
          rank += (w > gm) || (w == gm && q < pair);
        }
        if ((lane & 1) == 0) sh.gsort[warp][rank] = gm;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < SWARPS; ++w) {
          if (w == warp) continue;
          int lo = 0, hi = 16;  // entries of warp w that come before this value
#pragma unroll
          for (int it = 0; it < 5; ++it) {
            if (lo < hi) {
              const int mid = (lo + hi) >> 1;
              const float e = sh.gsort[w][mid];
              if (e > gm || (e == gm && w < warp)) lo = mid + 1;
              else hi = mid;
            }
          }
          rank += lo;
        }
        if ((lane & 1) == 0 && rank == kk - 1) sh.first_raw = gm;
        __syncthreads();
        const float raw = sh.first_raw;
        float hi = sh.gsort[0][0];
#pragma unroll
        for (int w = 1; w < SWARPS; ++w) hi = fmaxf(hi, sh.gsort[w][0]);
        base_key = ord_key(raw);
        const uint32_t span = ord_key(hi) > base_key ? ord_key(hi) - base_key : 0u;
        bin_shift = 0;
        while ((span >> bin_shift) >= (uint32_t)SBINS) ++bin_shift;
        te = lower_tau(raw, T);
      }
      // Hit units: their maximum reaches the bound (the raw maximum bounds the
      // penalised one from above).  Their 16 bytes and seen bits are kept for the
      // finish, which tests their elements.
      const float tcmp = fmaxf(te, -3.402823466e38f);  // excludes -inf
      uint32_t hu = 0;
#pragma unroll
      for (int j = 0; j < UPT; ++j) hu |= (uint32_t)(umax[j] >= tcmp) << j;
      if (hu) {
        int pos = atomicAdd(&sh.unit_n, __popc(hu));
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          if ((hu >> j) & 1u) {
            if (pos < UCAP) {
              const int k = tid + j * SNT;
              sh.udata[pos] = reinterpret_cast<const uint4*>(slot)[k];
              sh.uidx[pos] = ((u0 + k) << 8) | (int)sb[j];
            }
            ++pos;
          }
        }
      }
      // Histogram of the group values that can still raise the bound.
      if ((lane & 1) == 0) {
        const uint32_t k = ord_key(gm);
        if (gm >= te && k >= base_key)
          atomicAdd(&sh.bins[min((uint32_t)(SBINS - 1), (k - base_key) >> bin_shift)], 1u);
      }
      // The bound warp publishes a bound from the bins as they stand, before the
      // barrier so that its latency overlaps the other warps' passes (counts only
      // grow, so a partial histogram gives a valid, lower bound).  Every fourth
      // chunk only: the scan sits on each chunk's critical path, and a bound a few
      // chunks older keeps a few more units.
      if (warp == kBoundWarp && (c & 3) == 3) {
        __syncwarp();
        const float tb = hist_bound(sh.bins, base_key, bin_shift, kk, T);
        if (lane == 0) sh.te_pub = fmaxf(sh.te_pub, tb);
      }
      __syncthreads();  // the slot is consumed
      te = fmaxf(te, sh.te_pub);
      if (tid == kIssuer) issue_next();
    }
    // The final bound, from the complete bins.
    if (warp == kBoundWarp) {
      const float tb = hist_bound(sh.bins, base_key, bin_shift, kk, T);
      if (lane == 0) sh.te_pub = fmaxf(sh.te_pub, tb);
    }

    // 3. finish the row.
    if (rmx != rmx) atomicOr(&sh.err, 1 << ST_NAN);
    else if (rmx == PINF) atomicOr(&sh.err, 1 << ST_POSINF);
    rmx = warp_max_nan(rmx);
    if (lane == 0 && rmx == rmx) atomicMax(&sh.rmax_key, ord_key(rmx));
    if (tid == 0) bs.flag = 0;
    __syncthreads();
    const float tfin = fmaxf(fmaxf(te, sh.te_pub), -3.402823466e38f);  // final bound; excludes -inf
    const float uu = a.uniforms[row];
    const int nu = sh.unit_n;
    int status = sh.err ? first_err(sh.err) : ST_OK;
    bool general = status == ST_OK && a.force_slow;
    float* sval = reinterpret_cast<float*>(sh.work);
    int* sidx = reinterpret_cast<int*>(sh.work + 4 * SFIN);
    uint64_t* W = reinterpret_cast<uint64_t*>(sh.work + 8 * SFIN);
    float* fv = reinterpret_cast<float*>(W);
    int* fi = reinterpret_cast<int*>(sh.work + 12 * SFIN);
    // Kept list and leader_fast's key array, in the unit data (consumed by then).
    int* kidx = reinterpret_cast<int*>(sh.udata) + 2 * SFIN;
    float* kval = reinterpret_cast<float*>(sh.udata);
    int m = 0;
    if (status == ST_OK && !general) {
      // The elements of the hit units whose penalised score reaches the final
      // bound, tempered (elements outside the row were staged as -inf).  When the
      // list overflowed, the row is read again (from L2 or HBM) against that bound.
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
      if (nu > UCAP) {
        for (int64_t i = tid; i < V; i += SNT) {
          float x = Elem<TIn>::load(rowp + i);
          if (x >= tfin) {
            if ((bits[i >> 5] >> (i & 31)) & 1u) x = penalize(x, rp);
            if (x >= tfin) take((int)i, x);
          }
        }
      }
      for (int t = tid; t < (nu > UCAP ? 0 : nu); t += SNT) {
        const int ent = sh.uidx[t];
        const int uid = ent >> 8;
        float v[EPU];
        IO::load(reinterpret_cast<const TIn*>(sh.udata), t, v);
#pragma unroll
        for (int e = 0; e < EPU; ++e) {
          if (v[e] >= tfin) {
            const int i = uid * EPU + e - g.off_e;
            float x = v[e];
            if ((ent >> e) & 1) x = penalize(x, rp);
            if (x >= tfin) take(i, x);
          }
        }
      }
      if (bad) atomicOr(&sh.err, 1 << ST_POSINF);
      __syncthreads();
      m = bs.flag;
      if (sh.err) status = first_err(sh.err);
      __syncthreads();
      if (m > SFIN) general = status == ST_OK;
    }
    if (general && temper(key_to_float(sh.rmax_key), T) == PINF) {
      // A score may reach +inf only through the temperature: check every element.
      int inf = 0;
      for (int64_t i = tid; i < V; i += SNT) {
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
    if (status == ST_OK && !general && m <= 64 && !(a.out_dense && a.dense_mode != DENSE_NONE)) {
      // Common case: warp 0 finishes the row in registers while the other warps
      // start the next one (it touches nothing the next row's start uses).
      if (warp == 0) {
        int64_t tok = -1;
        const Kept kp = warp_finish<2>(a, fv, fi, m, uu, &tok, kidx, kval);
        const float Sf = fix_to_float(kp.tot);
        for (int j = lane; j < kp.n && j < a.out_cap; j += 32) {
          if (a.out_idx) a.out_idx[row * a.out_cap + j] = kidx[j];
          if (a.out_prob) a.out_prob[row * a.out_cap + j] = __fdiv_rn(sv_exp(__fsub_rn(kval[j], kp.M)), Sf);
          if (a.out_score) a.out_score[row * a.out_cap + j] = kval[j];
        }
        if (lane == 0) {
          a.out_token[row] = tok;
          if (a.out_count) a.out_count[row] = kp.n;
          if (a.out_status) a.out_status[row] = ST_OK;
          if (a.seen_bits && tok >= 0) atomicOr(&a.seen_bits[row * a.seen_bits_stride + (tok >> 5)], 1u << (tok & 31));
        }
      }
      continue;
    }
    Kept kept = {0, 0.0f, 0};
    int64_t token = -1;
    if (a.out_dense && a.dense_mode != DENSE_NONE && status == ST_OK && !general) {
      const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
      for (int64_t i = tid; i < V; i += SNT) a.out_dense[row * a.dense_stride + i] = dv;
      __syncthreads();
    }
    if (status == ST_OK && !general) {
      if (m <= 64) {
        // Few candidates: one warp finishes in registers.
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
        kept = leader_fast<SNT>(a, bs, fv, fi, m, sval, sidx, W, reinterpret_cast<uint64_t*>(sh.udata), kidx, kval);
        token = draw_kept<SNT>(bs, kidx, kval, kept, uu, reinterpret_cast<uint64_t*>(sh.work));
      }
      const float Sf = fix_to_float(kept.tot);
      for (int j = tid; j < kept.n; j += SNT) {
        const float p = __fdiv_rn(sv_exp(__fsub_rn(kval[j], kept.M)), Sf);
        if (j < a.out_cap) {
          if (a.out_idx) a.out_idx[row * a.out_cap + j] = kidx[j];
          if (a.out_prob) a.out_prob[row * a.out_cap + j] = p;
          if (a.out_score) a.out_score[row * a.out_cap + j] = kval[j];
        }
        if (a.out_dense && a.dense_mode != DENSE_NONE)
          a.out_dense[row * a.dense_stride + kidx[j]] = a.dense_mode == DENSE_SCORES ? kval[j] : p;
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
      kept = leader_slow<SNT, TIn, MODE_SAMPLE>(a, bs, sh.work, row, 0.0f, 0.0f, uu, &token, seen, emit);
    } else if (a.out_dense && a.dense_mode != DENSE_NONE) {
      const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
      for (int64_t i = tid; i < V; i += SNT) a.out_dense[row * a.dense_stride + i] = dv;
    }
    if (tid == 0) {
      a.out_token[row] = status == ST_OK ? token : -1;
      if (a.out_count) a.out_count[row] = kept.n;
      if (a.out_status) a.out_status[row] = status;
      if (status == ST_OK && a.seen_bits && token >= 0)
        atomicOr(&a.seen_bits[row * a.seen_bits_stride + (token >> 5)], 1u << (token & 31));
    }
    __syncthreads();
  }
}

template <typename TIn>
cudaError_t launch_stream_t(const RowArgs& a, size_t smem, cudaStream_t stream) {
  auto kern = stream_kernel<TIn>;
  static int configured[64] = {0};
  static int slots[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_limit_stream());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    slots[dev] = kCtasPerSm * sms;
    configured[dev] = 1;
  }
  const int grid = a.rows < slots[dev] ? a.rows : slots[dev];
  kern<<<grid, SNT, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

// Dynamic shared memory of the streaming kernel for a vocabulary, or 0 when it
// would not leave room for its CTAs per SM.
size_t stream_smem_bytes(int64_t vocab) {
  const size_t s = kStaticBytes + (size_t)SBUF * SCHUNK + bitmap_bytes(vocab);
  return s <= kSmemCap ? s : 0;
}

cudaError_t launch_stream(const RowArgs& a, size_t smem, cudaStream_t stream) {
  if (a.dtype == DT_F32) return launch_stream_t<float>(a, smem, stream);
  if (a.dtype == DT_F16) return launch_stream_t<__half>(a, smem, stream);
  return launch_stream_t<__nv_bfloat16>(a, smem, stream);
}

}  // namespace sv
