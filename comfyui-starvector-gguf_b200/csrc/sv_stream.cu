// sv_stream.cu -- the streaming row kernel (sm_100a): many independent rows.
//
// Persistent CTAs (three per SM) work through their rows one at a time.  A row's
// logits (and, ahead of them, its history ids) stream through a per-CTA ring of
// shared-memory slots filled by TMA bulk copies (cp.async.bulk, one mbarrier per
// slot); the ring runs ahead across row boundaries, so HBM keeps streaming while
// the CTA computes or finishes a row.
//
// Per row (runtime_shared.py:200-202):
//   1. the row's seen bitmap in shared memory, from the history;
//   2. per chunk, one pass: repetition penalty (:172-173), the candidate test
//      against the current lower bound tau of the row's k-th largest penalised
//      score, and the maxima of 128 lane groups.  The first chunk is read twice:
//      the exact k-th largest of its group maxima is the first bound.  Later group
//      maxima go into a 256-bin histogram over ordered float keys above that bound;
//      the highest bin edge with at least k group maxima at or above it is a valid,
//      tightening bound (group maxima of disjoint groups are distinct elements).
//      Candidates are tempered (:178-179) and appended to the row's list;
//   3. finish: candidates below the final bound are dropped, then the exact k-th
//      largest with ties (:180-181), top-p over the ascending (value, index) order
//      with exact fixed-point mass (:182-186) and the draw from the row's uniform.
//      A row with too many candidates (huge tie groups) takes the general path
//      over the whole row.
// No inter-CTA communication and no scratch memory in global memory.
#include <cuda_runtime.h>

#include "sv_block.cuh"
#include "sv_common.cuh"
#include "sv_internal.h"

namespace sv {

namespace {

constexpr int SNT = 256;               // threads per CTA
constexpr int SBUF = 3;                // ring slots
constexpr int SCHUNK = 16 * 1024;      // bytes per slot / chunk
constexpr int SCU = SCHUNK / 16;       // 16-byte units per chunk
constexpr int UPT = SCU / SNT;         // units per thread per chunk
constexpr int SG = 128;                // group maxima per chunk (groups of 2 lanes)
constexpr int SBINS = 256;             // bound histogram bins
constexpr int SCAP = kCandCap;         // candidates per row
constexpr int SFIN = 256;              // candidates the fast finish handles after pruning

struct __align__(16) StreamShared {
  unsigned long long mbar[SBUF];
  BlockScratch<SNT> bs;
  float gmax[SG];
  unsigned int bins[SBINS];
  unsigned int base_key;
  int bin_shift;
  float te_pub;  // bound published by warp 0 for the chunk after next
  int cand_n;
  int err;
  __align__(16) float cand_val[SCAP];
  int cand_idx[SCAP];
  __align__(16) unsigned char work[16 * SFIN];  // finish arrays / general-path scratch
};

constexpr size_t kStaticBytes = (sizeof(StreamShared) + 127) & ~size_t(127);

__host__ __device__ inline size_t bitmap_bytes(int64_t V) {
  return (((size_t)V + 31) / 32 * 4 + 16 + 127) & ~size_t(127);
}

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

// The bound from the histogram, computed by each warp on its own (identical in
// every warp): the highest bin b with at least kk group maxima in bins >= b gives
// key base + (b << shift).  Returns the lowered bound in the penalised domain.
__device__ __forceinline__ float hist_bound(const StreamShared& sh, int kk, float T) {
  const int lane = threadIdx.x & 31;
  uint32_t c[8], s = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    c[q] = sh.bins[lane * 8 + q];
    s += c[q];
  }
  uint32_t incl = s;  // count in bins of lanes >= lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += t;
  }
  int best = -1;
  if (incl >= (uint32_t)kk) {
    uint32_t above = incl - s;
    for (int q = 7; q >= 0; --q) {
      above += c[q];
      if (above >= (uint32_t)kk) {
        best = lane * 8 + q;
        break;
      }
    }
  }
  // The highest lane with a qualifying bin holds the answer.
  const unsigned m = __ballot_sync(0xffffffffu, best >= 0);
  const int src = m ? 31 - __clz(m) : 0;
  best = __shfl_sync(0xffffffffu, best, src);
  if (best < 0) return Elem<float>::neg_inf();
  const uint32_t k = sh.base_key + ((uint32_t)best << sh.bin_shift);
  return lower_tau(key_to_float(k), T);
}

// k-th largest (kk <= SG) of the SG group maxima by one warp: a bitwise radix
// select over ordered keys with ballots.  Returns the raw value (all lanes) and
// ORs NaN / +inf error bits into *err (lane 0).
__device__ __forceinline__ float warp_kth_of_groups(const float* g, int kk, int* err) {
  const int lane = threadIdx.x & 31;
  uint32_t k4[4];
  bool nan = false, pinf = false;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float v = g[lane * 4 + q];
    nan |= v != v;
    pinf |= v == __int_as_float(0x7f800000);
    k4[q] = ord_key(v);
  }
  nan = __any_sync(0xffffffffu, nan);
  pinf = __any_sync(0xffffffffu, pinf);
  uint32_t res = 0;
  for (int b = 31; b >= 0; --b) {
    const uint32_t c = res | (1u << b);
    const int n = __popc(__ballot_sync(0xffffffffu, k4[0] >= c)) + __popc(__ballot_sync(0xffffffffu, k4[1] >= c)) +
                  __popc(__ballot_sync(0xffffffffu, k4[2] >= c)) + __popc(__ballot_sync(0xffffffffu, k4[3] >= c));
    if (n >= kk) res = c;
  }
  if (lane == 0 && (nan || pinf)) atomicOr(err, 1 << (nan ? ST_NAN : ST_POSINF));
  return key_to_float(res);
}

template <typename TIn>
__global__ void __launch_bounds__(SNT, 3) stream_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StreamShared& sh = *reinterpret_cast<StreamShared*>(smem_raw);
  BlockScratch<SNT>& bs = sh.bs;
  unsigned char* ring = smem_raw + kStaticBytes;
  uint32_t* bits = reinterpret_cast<uint32_t*>(ring + (size_t)SBUF * SCHUNK);
  constexpr int ES = Elem<TIn>::kSize;
  constexpr int EPU = 16 / ES;
  using IO = UnitIO<TIn>;
  const int tid = threadIdx.x, lane = tid & 31;
  const float NEG = Elem<float>::neg_inf();
  const int64_t V = a.vocab;
  const int nw = (int)((V + 31) >> 5);
  const float rp = a.rep_penalty, T = a.temperature;
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
  int64_t issued = 0;
  if (tid == 0) {
    for (int s = 0; s < SBUF; ++s) mbar_init(&sh.mbar[s], 1);
    mbar_init_fence();
    sh.err = 0;
  }
  __syncthreads();
  auto issue_next = [&]() {  // thread 0, after a block barrier
    if (irow >= a.rows) return;
    fence_proxy_async_smem();
    const int s = (int)(issued % SBUF);
    unsigned char* slot = ring + (size_t)s * SCHUNK;
    if (ic < 0) {
      mbar_expect_tx(&sh.mbar[s], (uint32_t)hbytes);
      bulk_g2s(slot, reinterpret_cast<const unsigned char*>(a.hist) + (size_t)irow * a.hist_stride * idb,
               (uint32_t)hbytes, &sh.mbar[s]);
    } else {
      issue_chunk(ig, ic, slot, &sh.mbar[s]);
    }
    ++issued;
    if (++ic == ig.nch) {
      ic = stage_ids ? -1 : 0;
      irow += step;
      if (irow < a.rows) ig = row_geom<TIn>(a, irow);
    }
  };
  if (tid == 0)
    for (int s = 0; s < SBUF; ++s) issue_next();

  int64_t consumed = 0;  // slots consumed so far (all threads)
  for (int64_t row = first; row < a.rows; row += step) {
    const RowGeom g = row_geom<TIn>(a, row);
    const TIn* rowp = reinterpret_cast<const TIn*>(a.logits) + row * a.row_stride;
    const bool aligned = g.off_e == 0;
    // 1. seen bitmap of the row.
    for (int w = tid; w < nw + 4; w += SNT) bits[w] = 0;
    for (int b = tid; b < SBINS; b += SNT) sh.bins[b] = 0;
    if (tid == 0) {
      sh.cand_n = 0;
      sh.te_pub = NEG;
    }
    __syncthreads();
    int local_err = 0;
    if (ids_kind) {
      const int64_t L = hist_length(a, row);
      const void* src;
      int64_t s = -1;
      if (stage_ids) {
        s = consumed % SBUF;
        if (!mbar_wait(&sh.mbar[s], (uint32_t)((consumed / SBUF) & 1))) local_err |= 1 << ST_TIMEOUT;
        src = ring + (size_t)s * SCHUNK;
      } else {
        src = reinterpret_cast<const unsigned char*>(a.hist) + (size_t)row * a.hist_stride * idb;
      }
      constexpr int U = 8;
      for (int64_t base = 0; base < L; base += (int64_t)SNT * U) {
        int64_t id[U];
#pragma unroll
        for (int q = 0; q < U; ++q) {
          const int64_t j = base + tid + (int64_t)q * SNT;
          id[q] = j >= L ? 0
                         : (idb == 4 ? (int64_t) reinterpret_cast<const int32_t*>(src)[j]
                                     : reinterpret_cast<const int64_t*>(src)[j]);
        }
#pragma unroll
        for (int q = 0; q < U; ++q) {
          const int64_t j = base + tid + (int64_t)q * SNT;
          if (j >= L) continue;
          if (id[q] < 0 || id[q] >= V) {
            local_err |= 1 << ST_HISTORY;
            continue;
          }
          const uint32_t b = 1u << (id[q] & 31);
          uint32_t* w = &bits[id[q] >> 5];
          if (!(*w & b)) atomicOr(w, b);  // repeated ids mostly find their bit set
        }
      }
      if (stage_ids) {
        ++consumed;
        __syncthreads();  // the ids slot is consumed
        if (tid == 0) issue_next();
      }
    } else if (a.hist_kind == HIST_BITS32) {
      const uint32_t* hb = reinterpret_cast<const uint32_t*>(a.hist) + row * a.hist_stride;
      for (int w = tid; w < nw; w += SNT) {
        uint32_t v = hb[w];
        if (w == nw - 1 && (V & 31)) v &= (1u << (V & 31)) - 1u;
        bits[w] = v;
      }
    } else if (a.hist_kind == HIST_MASK8) {
      for (int64_t i = tid; i < V; i += SNT)
        if (seen_global(a, row, i)) atomicOr(&bits[i >> 5], 1u << (i & 31));
    }
    if (local_err) atomicOr(&sh.err, local_err);
    __syncthreads();

    // 2. chunks.
    float te = NEG;
    for (int c = 0; c < g.nch; ++c, ++consumed) {
      const int s = (int)(consumed % SBUF);
      TIn* slot = reinterpret_cast<TIn*>(ring + (size_t)s * SCHUNK);
      if (!mbar_wait(&sh.mbar[s], (uint32_t)((consumed / SBUF) & 1))) atomicOr(&sh.err, 1 << ST_TIMEOUT);
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
      const bool two_pass = c == 0;
      // Seen-bit lookup: for aligned rows each of this thread's units sits at a fixed
      // bit offset in consecutive bitmap words.
      const int ubase = u0 + tid;
      for (int pass = two_pass ? 0 : 1; pass < 2; ++pass) {
        const bool collect = pass == 1;
        const bool groups = !(collect && two_pass);
        // One compare excludes -inf and keeps every finite value >= te.
        const float tcmp = fmaxf(te, -3.402823466e38f);
        float v[UPT][EPU];
        uint32_t sb[UPT];
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          const int k = tid + j * SNT;
          if (k < un) {
            IO::load(slot, k, v[j]);
          } else {
#pragma unroll
            for (int e = 0; e < EPU; ++e) v[j][e] = NEG;
          }
        }
        if (aligned) {
          const int shift = (ubase * EPU) & 31;
#pragma unroll
          for (int j = 0; j < UPT; ++j) {
            const int k = tid + j * SNT;
            sb[j] = k < un ? (bits[((ubase + j * SNT) * EPU) >> 5] >> shift) & ((1u << EPU) - 1u) : 0u;
          }
        } else {
#pragma unroll
          for (int j = 0; j < UPT; ++j) {
            const int k = tid + j * SNT;
            sb[j] = k < un ? unit_bits(bits, (int64_t)(u0 + k) * EPU - g.off_e, EPU, V) : 0u;
          }
        }
        float tmax = NEG;
        uint32_t hits = 0;
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          if (sb[j]) {
#pragma unroll
            for (int e = 0; e < EPU; ++e)
              if ((sb[j] >> e) & 1u) v[j][e] = penalize(v[j][e], rp);
          }
#pragma unroll
          for (int e = 0; e < EPU; ++e) {
            if (groups) tmax = max_nan(tmax, v[j][e]);
            if (collect) hits |= (uint32_t)(v[j][e] >= tcmp) << (j * EPU + e);
          }
        }
        if (collect && __any_sync(0xffffffffu, hits != 0)) {
          // One atomic per warp: lanes' hit counts are scanned, then written.
          const int cnt = __popc(hits);
          int incl = cnt;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
          }
          int base = 0;
          if (lane == 31) base = atomicAdd(&sh.cand_n, incl);
          base = __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
          // Hits are re-read from the slot (a register array indexed at run time would
          // live in local memory); a hit is a finite element inside the row.
          while (hits) {
            const int q = __ffs(hits) - 1;
            hits &= hits - 1;
            const int k = tid + (q / EPU) * SNT, e = q % EPU;
            const int i = (u0 + k) * EPU + e - g.off_e;
            float x = Elem<TIn>::to_f(slot[k * EPU + e]);
            if ((bits[i >> 5] >> (i & 31)) & 1u) x = penalize(x, rp);
            if (base < SCAP) {
              sh.cand_val[base] = temper(x, T);
              sh.cand_idx[base] = i;
            }
            ++base;
          }
        }
        if (groups) {
          tmax = max_nan(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
          if (two_pass) {
            // First chunk: the exact k-th largest of its group maxima anchors the bins.
            if ((tid & 1) == 0) sh.gmax[tid >> 1] = tmax;
            __syncthreads();
            if (tid < 32) {
              const float raw = warp_kth_of_groups(sh.gmax, kk, &sh.err);
              float top = NEG;
#pragma unroll
              for (int q = 0; q < 4; ++q) top = fmaxf(top, sh.gmax[lane * 4 + q]);
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
              if (lane == 0) {
                const uint32_t base = ord_key(raw);
                const uint32_t span = ord_key(top) > base ? ord_key(top) - base : 0u;
                int shf = 0;
                while ((span >> shf) >= (uint32_t)SBINS) ++shf;
                sh.base_key = base;
                sh.bin_shift = shf;
                sh.te_pub = lower_tau(raw, T);
              }
            }
            __syncthreads();
            te = sh.te_pub;
          }
          if ((tid & 1) == 0) {
            if (tmax != tmax) atomicOr(&sh.err, 1 << ST_NAN);
            else if (tmax == __int_as_float(0x7f800000)) atomicOr(&sh.err, 1 << ST_POSINF);
            else {
              const uint32_t k = ord_key(tmax);
              if (k >= sh.base_key) atomicAdd(&sh.bins[min((uint32_t)(SBINS - 1), (k - sh.base_key) >> sh.bin_shift)], 1u);
            }
          }
        }
      }
      __syncthreads();  // the slot is consumed; the bins hold this chunk's maxima
      // The bound published during the previous chunk (bins complete up to the chunk
      // before it); warp 0 then publishes one from the bins complete up to this chunk,
      // read after the next chunk's barrier.
      te = fmaxf(te, sh.te_pub);
      if (tid < 32) {
        const float tb = hist_bound(sh, kk, T);
        __syncwarp();
        if (lane == 0) sh.te_pub = tb;
      }
      if (tid == 0) issue_next();
    }

    // 3. finish the row.
    const float uu = a.uniforms[row];
    int status = sh.err ? first_err(sh.err) : ST_OK;
    const int n = sh.cand_n;
    if (status == ST_OK && n == 0) status = ST_ALLNEGINF;
    Kept kept = {0, 0.0f, 0};
    int64_t token = -1;
    bool general = status == ST_OK && (a.force_slow || n > SCAP);
    float* sval = reinterpret_cast<float*>(sh.work);
    int* sidx = reinterpret_cast<int*>(sh.work + 4 * SFIN);
    uint64_t* W = reinterpret_cast<uint64_t*>(sh.work + 8 * SFIN);
    float* fv = reinterpret_cast<float*>(W);
    int* fi = reinterpret_cast<int*>(sh.work + 12 * SFIN);
    int m = 0;
    if (status == ST_OK && !general) {
      // Drop candidates below the final bound (monotone in the tempered domain).
      const float tft = te == NEG ? NEG : __fdiv_rn(te, T);
      if (tid == 0) bs.flag = 0;
      __syncthreads();
      for (int t = tid; t < n; t += SNT) {
        const float v = sh.cand_val[t];
        if (v >= tft) {
          const int at = atomicAdd(&bs.flag, 1);
          if (at < SFIN) {
            fv[at] = v;
            fi[at] = sh.cand_idx[t];
          }
        }
      }
      __syncthreads();
      m = bs.flag;
      __syncthreads();
      if (m > SFIN) general = true;
    }
    if (a.out_dense && a.dense_mode != DENSE_NONE && status == ST_OK && !general) {
      const float dv = a.dense_mode == DENSE_SCORES ? NEG : 0.0f;
      for (int64_t i = tid; i < V; i += SNT) a.out_dense[row * a.dense_stride + i] = dv;
      __syncthreads();
    }
    if (status == ST_OK && !general) {
      kept = leader_fast<SNT>(a, bs, fv, fi, m, sval, sidx, W, reinterpret_cast<uint64_t*>(sh.cand_val),
                              sh.cand_idx, sh.cand_val);
      token = draw_kept<SNT>(bs, sh.cand_idx, sh.cand_val, kept, uu, reinterpret_cast<uint64_t*>(sh.work));
      const float Sf = fix_to_float(kept.tot);
      for (int j = tid; j < kept.n; j += SNT) {
        const float p = __fdiv_rn(sv_exp(__fsub_rn(sh.cand_val[j], kept.M)), Sf);
        if (j < a.out_cap) {
          if (a.out_idx) a.out_idx[row * a.out_cap + j] = sh.cand_idx[j];
          if (a.out_prob) a.out_prob[row * a.out_cap + j] = p;
          if (a.out_score) a.out_score[row * a.out_cap + j] = sh.cand_val[j];
        }
        if (a.out_dense && a.dense_mode != DENSE_NONE)
          a.out_dense[row * a.dense_stride + sh.cand_idx[j]] = a.dense_mode == DENSE_SCORES ? sh.cand_val[j] : p;
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
      sh.err = 0;
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
    slots[dev] = 3 * sms;
    configured[dev] = 1;
  }
  const int grid = a.rows < slots[dev] ? a.rows : slots[dev];
  kern<<<grid, SNT, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

// Dynamic shared memory of the streaming kernel for a vocabulary, or 0 when it
// would not leave room for three CTAs per SM.
size_t stream_smem_bytes(int64_t vocab) {
  const size_t s = kStaticBytes + (size_t)SBUF * SCHUNK + bitmap_bytes(vocab);
  return s <= 74 * 1024 ? s : 0;
}

cudaError_t launch_stream(const RowArgs& a, size_t smem, cudaStream_t stream) {
  if (a.dtype == DT_F32) return launch_stream_t<float>(a, smem, stream);
  if (a.dtype == DT_F16) return launch_stream_t<__half>(a, smem, stream);
  return launch_stream_t<__nv_bfloat16>(a, smem, stream);
}

}  // namespace sv
