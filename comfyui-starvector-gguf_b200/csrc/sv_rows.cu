// sv_rows.cu -- the cluster row kernel (sm_100a): few rows, low latency, beams.
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
//   3. The leader (cluster rank 0) finishes the row from the candidates: exact
//      top-k threshold with ties (runtime_shared.py:180-181), top-p over the
//      ascending (value, index) order with exact fixed-point mass (:182-186), the
//      draw (sample mode) or the kept list for the beam merge (beam mode).
//      More than kCandCap candidates (huge tie groups) take the general path that
//      re-reads the row from global memory and handles the tie group
//      arithmetically.
//   4. Beam mode: the last beam leader to finish (atomic counter, no waiting)
//      merges the beams: + running scores, softmax over beams*V, count_nonzero,
//      draws without replacement (runtime_shared.py:231-237).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "sv_block.cuh"
#include "sv_common.cuh"
#include "sv_internal.h"

namespace cg = cooperative_groups;

namespace sv {

namespace {

constexpr int NT = kThreads;
constexpr int CAP = kCandCap;

struct __align__(16) Shared {
  unsigned long long mbar[kChunks];
  BlockScratch<NT> bs;
  float gmax[kGroups];
  float gmax2[kGroups];
  float red_max[kMaxCluster];
  unsigned long long red_sum[kMaxCluster];
  int cand_n;
  int err;
  float tau_eff;
  __align__(16) float cand_val[CAP];
  int cand_idx[CAP];
};

// Named barrier 1: warp 0 arrives (producer), the other warps wait (consumers).
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ T* remote(cg::cluster_group& cl, T* p, int rank) {
  return cl.map_shared_rank(p, rank);
}

// ------------------------------------------------------------------ beam merge
// A NaN flattened score (runtime_shared.py:231): a NaN running score, or +inf
// added to the -inf of a beam's entries outside its kept list.
__device__ __forceinline__ bool running_gives_nan(float rs, int count, int64_t vocab) {
  return rs != rs || (rs == __int_as_float(0x7f800000) && (int64_t)count < vocab);
}

// Runs in the last beam leader to finish.  Entries of all beams in flattened
// (beam-major, index-ascending) order.
__device__ void beam_merge(const RowArgs& a, Shared& sh, unsigned char* regA) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int B = a.rows;
  const BeamWsHeader* hdr = reinterpret_cast<const BeamWsHeader*>(a.ws);
  const int* kidx0 = reinterpret_cast<const int*>(a.ws + sizeof(BeamWsHeader));
  const float* kval0 = reinterpret_cast<const float*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 4);
  uint64_t* Wg = reinterpret_cast<uint64_t*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 8);
  __shared__ int offs[kMaxBeams + 1];
  __shared__ int picked[2 * kMaxBeams];
  __shared__ float uni[64];             // the draws' uniforms (num_picks <= 64)
  __shared__ float run[kMaxBeams];      // running scores
  BlockScratch<NT>& bs = sh.bs;
  // Loaded ahead: the draws are sequential and must not wait on memory each.
  if (tid < a.npick) uni[tid] = a.uniforms[tid];
  if (tid < B) run[tid] = a.running[tid];
  if (tid == 0) {
    int st = ST_OK, o = 0;
    bool nan_score = false;
    for (int b = 0; b < B; ++b) {
      const int s = __ldcg(&hdr->status[b]);
      const int c = __ldcg(&hdr->count[b]);
      if (s != ST_OK && st == ST_OK) st = s;
      nan_score |= running_gives_nan(a.running[b], c, a.vocab);
      offs[b] = o;
      o += c;
    }
    offs[B] = o;
    bs.flag = st == ST_OK && nan_score ? ST_NAN : st;
  }
  __syncthreads();
  const int st = bs.flag;
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
  // Scores (+ running score) and flattened ids staged in shared memory in one pass
  // when they fit.
  const bool in_smem = K <= 1024;
  float* es = reinterpret_cast<float*>(regA);
  uint64_t* W = in_smem ? reinterpret_cast<uint64_t*>(regA + 4096) : Wg;
  int64_t* ef = reinterpret_cast<int64_t*>(regA + 12288);  // K <= 512 only
  const bool ids_smem = K <= 512;
  auto score_of = [&](int e, int b) -> float {
    return in_smem ? es[e] : __fadd_rn(__ldcg(&kval0[(size_t)b * a.ws_cap + (e - offs[b])]), run[b]);
  };
  if (in_smem) {
    for (int e = tid; e < K; e += NT) {
      const int b = beam_of(e);
      es[e] = __fadd_rn(__ldcg(&kval0[(size_t)b * a.ws_cap + (e - offs[b])]), run[b]);
      if (ids_smem) ef[e] = (int64_t)b * a.vocab + __ldcg(&kidx0[(size_t)b * a.ws_cap + (e - offs[b])]);
    }
    __syncthreads();
  }
  float mx = Elem<float>::neg_inf();
  for (int e = tid; e < K; e += NT) mx = max_nan(mx, score_of(e, beam_of(e)));
  const float Ms = block_max_nan<NT>(bs, mx);
  if (Ms == __int_as_float(0x7f800000) || Ms == Elem<float>::neg_inf()) {
    if (tid == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = Ms > 0.0f ? ST_POSINF : ST_ALLNEGINF;
    }
    return;
  }
  uint64_t ls = 0;
  for (int e = tid; e < K; e += NT) {
    const float s = score_of(e, beam_of(e));
    W[e] = fixw(sv_exp(__fsub_rn(s, Ms)));
    ls += W[e];
  }
  const uint64_t tot = block_sum_u64<NT>(bs, ls);
  const float Sf = fix_to_float(tot);
  int nz = 0;
  for (int e = tid; e < K; e += NT) {
    const int b = beam_of(e);
    const float p = __fdiv_rn(sv_exp(__fsub_rn(score_of(e, b), Ms)), Sf);
    nz += p > 0.0f;
    const int j = e - offs[b];
    if (a.out_prob && j < a.out_cap) a.out_prob[(size_t)b * a.out_cap + j] = p;
  }
  const int nnz = block_sum_int<NT>(bs, nz);
  const int n = a.npick < nnz ? a.npick : nnz;
  __syncthreads();
  if (tid < 32) {
    const int seg = (K + 31) / 32;
    const int e0 = lane * seg, e1 = min(K, e0 + seg);
    uint64_t mysum = 0;
    for (int e = e0; e < e1; ++e) mysum += W[e];
    // Inclusive prefix of the lanes' segment sums and the total, scanned once and
    // then updated as picks remove weight.
    uint64_t incl = mysum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    uint64_t total = __shfl_sync(0xffffffffu, incl, 31);
    for (int j = 0; j < n; ++j) {
      int pick = -1;
      if (total > 0) {
        const uint64_t t = mulfloor(total, uni[j]);
        const uint64_t excl = incl - mysum;
        const bool own = mysum > 0 && excl <= t && t < incl;
        const unsigned bm = __ballot_sync(0xffffffffu, own);
        const int o = __ffs(bm) - 1;
        uint64_t w = 0;
        if (lane == o) {
          // The whole segment without an early exit: its weights load together.
          uint64_t c = excl;
#pragma unroll 8
          for (int e = e0; e < e1; ++e) {
            const uint64_t we = W[e];
            c += we;
            if (pick < 0 && c > t) {
              pick = e;
              w = we;
            }
          }
          mysum -= w;
          W[pick] = 0;
        }
        pick = __shfl_sync(0xffffffffu, pick, o);
        w = __shfl_sync(0xffffffffu, w, o);
        if (lane >= o) incl -= w;
        total -= w;
      } else {
        // No fixed-point mass left: the largest remaining nonzero probability.
        float best = -1.0f;
        int be = K;
        for (int e = e0; e < e1; ++e) {
          bool done = false;
          for (int q = 0; q < j; ++q) done |= picked[q] == e;
          if (done) continue;
          const float p = __fdiv_rn(sv_exp(__fsub_rn(score_of(e, beam_of(e)), Ms)), Sf);
          if (p > 0.0f && (p > best || (p == best && e < be))) {
            best = p;
            be = e;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          float ob = __shfl_xor_sync(0xffffffffu, best, o);
          int oe = __shfl_xor_sync(0xffffffffu, be, o);
          if (ob > best || (ob == best && oe < be)) {
            best = ob;
            be = oe;
          }
        }
        pick = be;
      }
      if (lane == 0) picked[j] = pick;
      __syncwarp();
    }
    // The picks' outputs, one lane each, off the draws' dependency chain.
    for (int j = lane; j < n; j += 32) {
      const int pick = picked[j];
      const int b = beam_of(pick);
      a.out_picks[j] = in_smem && ids_smem ? ef[pick]
                                           : (int64_t)b * a.vocab + __ldcg(&kidx0[(size_t)b * a.ws_cap + (pick - offs[b])]);
      a.out_pick_scores[j] = score_of(pick, b);
    }
    if (lane == 0) {
      *a.out_npicks = n;
      a.out_status[0] = ST_OK;
    }
  }
}

// Small kept lists (two beams of top-k 50 fit: 64 slots a beam): warp 0 alone
// merges in registers, with no block barrier.  Lane L holds beam b = L / (32 / B) and slots
// (L % (32 / B)) * kMergeR .. + kMergeR - 1 of that beam's kept list, so lane order
// then slot order is the flattened (beam-major, index-ascending) order of
// runtime_shared.py:231 and slots past a beam's count carry no weight.  The counts,
// statuses and slots are loaded together, in one round trip to L2.  Returns false,
// having written nothing, when a beam keeps more entries than its lanes hold; the
// block merge then runs.  Same arithmetic as beam_merge, element for element.
constexpr int kMergeR = 4;

// Loads issued where they are written: the merge's inputs are all requested in one
// round trip before the first use, and the compiler neither sinks nor splits them.
__device__ __forceinline__ float ld_now(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_now(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool beam_merge_warp(const RowArgs& a) {
  const int lane = threadIdx.x & 31;
  const int B = a.rows;
  const int LB = 32 / B;  // lanes per beam (B <= kMaxBeams = 32)
  const int b = lane / LB;
  const bool act = b < B;
  const int j0 = (lane - b * LB) * kMergeR;
  const BeamWsHeader* hdr = reinterpret_cast<const BeamWsHeader*>(a.ws);
  const int* kidx0 = reinterpret_cast<const int*>(a.ws + sizeof(BeamWsHeader));
  const float* kval0 = reinterpret_cast<const float*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 4);
  const float NEG = Elem<float>::neg_inf();
  int cnt = 0, stt = ST_OK;
  float runb = 0.0f;
  float s[kMergeR];  // kept log-probability + running score
  int ki[kMergeR];
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    s[r] = 0.0f;
    ki[r] = 0;
  }
  float u0 = 0.0f, u1 = 0.0f;
  if (lane < a.npick) u0 = ld_now(&a.uniforms[lane]);
  if (lane + 32 < a.npick) u1 = ld_now(&a.uniforms[lane + 32]);
  if (act) {
    cnt = ld_now(&hdr->count[b]);
    stt = ld_now(&hdr->status[b]);
    runb = ld_now(&a.running[b]);
#pragma unroll
    for (int r = 0; r < kMergeR; ++r) {
      const int j = j0 + r;
      if (j < a.ws_cap) {
        s[r] = ld_now(&kval0[(size_t)b * a.ws_cap + j]);
        ki[r] = ld_now(&kidx0[(size_t)b * a.ws_cap + j]);
      }
    }
  }
  if (__ballot_sync(0xffffffffu, act && cnt > LB * kMergeR)) return false;
  const unsigned bad = __ballot_sync(0xffffffffu, act && stt != ST_OK);
  const bool nan_score = __any_sync(0xffffffffu, act && running_gives_nan(runb, cnt, a.vocab));
  const int st = bad ? __shfl_sync(0xffffffffu, stt, __ffs(bad) - 1) : (nan_score ? ST_NAN : ST_OK);
  const int K = warp_sum_int(act && lane == b * LB ? cnt : 0);
  if (st != ST_OK || K == 0) {
    if (lane == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = st != ST_OK ? st : ST_ALLNEGINF;
    }
    return true;
  }
  unsigned valid = 0;
  float mx = NEG;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    const bool v = act && j0 + r < cnt;
    valid |= (unsigned)v << r;
    s[r] = __fadd_rn(s[r], runb);
    if (v) mx = max_nan(mx, s[r]);
  }
  const float Ms = warp_max_nan(mx);
  if (Ms == __int_as_float(0x7f800000) || Ms == NEG) {
    if (lane == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = Ms > 0.0f ? ST_POSINF : ST_ALLNEGINF;
    }
    return true;
  }
  uint64_t W[kMergeR];
  float ex[kMergeR];
  uint64_t lsum = 0;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    const bool v = (valid >> r) & 1u;
    ex[r] = v ? sv_exp(__fsub_rn(s[r], Ms)) : 0.0f;
    W[r] = fixw(ex[r]);
    lsum += W[r];
  }
  const uint64_t tot = warp_sum_u64(lsum);
  const float Sf = fix_to_float(tot);
  int nz = 0;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    if (!((valid >> r) & 1u)) continue;
    const float p = __fdiv_rn(ex[r], Sf);
    nz += p > 0.0f;
    const int j = j0 + r;
    if (a.out_prob && j < a.out_cap) a.out_prob[(size_t)b * a.out_cap + j] = p;
  }
  const int nnz = warp_sum_int(nz);
  const int n = a.npick < nnz ? a.npick : nnz;
  uint64_t lexcl = warp_incl_scan_u64(lsum) - lsum;
  uint64_t total = tot;
  unsigned taken = 0;
  for (int j = 0; j < n; ++j) {
    const float uj = __shfl_sync(0xffffffffu, j < 32 ? u0 : u1, j & 31);
    int owner, rs = -1;
    if (total > 0) {
      // The element whose fixed-point interval holds floor(total * u): its lane
      // first, then its slot by a walk of the lane's weights.
      const uint64_t t = mulfloor(total, uj);
      const bool own = lsum > 0 && lexcl <= t && t < lexcl + lsum;
      owner = __ffs(__ballot_sync(0xffffffffu, own)) - 1;
      uint64_t w = 0;
      if (lane == owner) {
        uint64_t c = lexcl;
#pragma unroll
        for (int r = 0; r < kMergeR; ++r) {
          c += W[r];
          if (rs < 0 && c > t) rs = r;
        }
#pragma unroll
        for (int r = 0; r < kMergeR; ++r)
          if (r == rs) {
            w = W[r];
            W[r] = 0;
          }
        lsum -= w;
      }
      w = __shfl_sync(0xffffffffu, w, owner);
      if (lane > owner) lexcl -= w;
      total -= w;
    } else {
      // No fixed-point mass left: the largest remaining nonzero probability,
      // ties to the lowest flattened position.
      float best = -1.0f;
      int be = 0x7fffffff;
#pragma unroll
      for (int r = 0; r < kMergeR; ++r) {
        if (!((valid >> r) & 1u) || ((taken >> r) & 1u)) continue;
        const float p = __fdiv_rn(sv_exp(__fsub_rn(s[r], Ms)), Sf);
        if (p > 0.0f && p > best) {
          best = p;
          be = lane * kMergeR + r;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
      owner = be / kMergeR;
      rs = be - owner * kMergeR;
    }
    if (lane == owner) {
      // The pick's outputs from the owner's registers.
#pragma unroll
      for (int r = 0; r < kMergeR; ++r)
        if (r == rs) {
          taken |= 1u << r;
          a.out_picks[j] = (int64_t)b * a.vocab + ki[r];
          a.out_pick_scores[j] = s[r];
        }
    }
  }
  if (lane == 0) {
    *a.out_npicks = n;
    a.out_status[0] = ST_OK;
  }
  return true;
}

// The same merge spread over the block when a beam keeps more than its lanes of
// one warp hold (eight beams of top-k 50): thread t holds beam b = t / (NT / B)
// and slots (t % (NT / B)) * kMergeR .. + kMergeR - 1, so thread order then slot
// order is again the flattened order.  Every input is requested in one round trip;
// the reductions take one barrier each and every draw one.  Returns false, having
// written nothing, when a beam keeps more entries than its threads hold.
struct MergeShared {
  float uni[64];
  int stat[kMaxBeams];
  int first_bad, flags, K;
  float wmax[NT / 32];
  unsigned long long wsum[NT / 32];
  int wnz[NT / 32];
  unsigned long long pick_w[2];
  float fb_p[2][NT / 32];
  int fb_e[2][NT / 32];
};

__device__ bool beam_merge_block(const RowArgs& a) {
  __shared__ MergeShared m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = NT / 32;
  const int B = a.rows;
  const int TB = NT / B;  // threads per beam (B <= kMaxBeams)
  const int b = tid / TB;
  const bool act = b < B;
  const bool lead = act && tid == b * TB;
  const int j0 = (tid - b * TB) * kMergeR;
  const BeamWsHeader* hdr = reinterpret_cast<const BeamWsHeader*>(a.ws);
  const int* kidx0 = reinterpret_cast<const int*>(a.ws + sizeof(BeamWsHeader));
  const float* kval0 = reinterpret_cast<const float*>(a.ws + sizeof(BeamWsHeader) + (size_t)B * a.ws_cap * 4);
  const float NEG = Elem<float>::neg_inf();
  int cnt = 0, stt = ST_OK;
  float runb = 0.0f, uv = 0.0f;
  float s[kMergeR];
  int ki[kMergeR];
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    s[r] = 0.0f;
    ki[r] = 0;
  }
  if (tid < a.npick) uv = ld_now(&a.uniforms[tid]);
  if (act) {
    cnt = ld_now(&hdr->count[b]);
    stt = ld_now(&hdr->status[b]);
    runb = ld_now(&a.running[b]);
#pragma unroll
    for (int r = 0; r < kMergeR; ++r) {
      const int j = j0 + r;
      if (j < a.ws_cap) {
        s[r] = ld_now(&kval0[(size_t)b * a.ws_cap + j]);
        ki[r] = ld_now(&kidx0[(size_t)b * a.ws_cap + j]);
      }
    }
  }
  if (tid == 0) {
    m.first_bad = B;
    m.flags = 0;
    m.K = 0;
  }
  __syncthreads();
  if (tid < a.npick) m.uni[tid] = uv;
  if (lead) {
    m.stat[b] = stt;
    if (stt != ST_OK) atomicMin(&m.first_bad, b);
    if (running_gives_nan(runb, cnt, a.vocab)) atomicOr(&m.flags, 2);
    atomicAdd(&m.K, cnt);
  }
  if (act && cnt > TB * kMergeR) atomicOr(&m.flags, 1);
  __syncthreads();
  const int flags = m.flags;
  if (flags & 1) return false;
  const int st = m.first_bad < B ? m.stat[m.first_bad] : ((flags & 2) ? ST_NAN : ST_OK);
  if (st != ST_OK || m.K == 0) {
    if (tid == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = st != ST_OK ? st : ST_ALLNEGINF;
    }
    return true;
  }
  unsigned valid = 0;
  float mx = NEG;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    const bool v = act && j0 + r < cnt;
    valid |= (unsigned)v << r;
    s[r] = __fadd_rn(s[r], runb);
    if (v) mx = max_nan(mx, s[r]);
  }
  mx = warp_max_nan(mx);
  if (lane == 0) m.wmax[warp] = mx;
  __syncthreads();
  float Ms = m.wmax[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) Ms = max_nan(Ms, m.wmax[w]);
  if (Ms == __int_as_float(0x7f800000) || Ms == NEG) {
    if (tid == 0) {
      *a.out_npicks = 0;
      a.out_status[0] = Ms > 0.0f ? ST_POSINF : ST_ALLNEGINF;
    }
    return true;
  }
  uint64_t W[kMergeR], excl[kMergeR];
  float ex[kMergeR];
  uint64_t lsum = 0;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    ex[r] = ((valid >> r) & 1u) ? sv_exp(__fsub_rn(s[r], Ms)) : 0.0f;
    W[r] = fixw(ex[r]);
    excl[r] = lsum;
    lsum += W[r];
  }
  const uint64_t lincl = warp_incl_scan_u64(lsum);
  if (lane == 31) m.wsum[warp] = lincl;
  __syncthreads();
  uint64_t total = 0, wbase = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const uint64_t v = m.wsum[w];
    if (w < warp) wbase += v;
    total += v;
  }
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) excl[r] += wbase + lincl - lsum;
  const float Sf = fix_to_float(total);
  int nz = 0;
#pragma unroll
  for (int r = 0; r < kMergeR; ++r) {
    const bool v = (valid >> r) & 1u;
    const float p = __fdiv_rn(ex[r], Sf);
    nz += __popc(__ballot_sync(0xffffffffu, v && p > 0.0f));
    const int j = j0 + r;
    if (v && a.out_prob && j < a.out_cap) a.out_prob[(size_t)b * a.out_cap + j] = p;
  }
  if (lane == 0) m.wnz[warp] = nz;
  __syncthreads();
  int nnz = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) nnz += m.wnz[w];
  const int n = a.npick < nnz ? a.npick : nnz;
  unsigned taken = 0;
  for (int j = 0; j < n; ++j) {
    const int q = j & 1;  // double-buffered: a slot is rewritten two draws later
    int rs = -1;
    if (total > 0) {
      // The element whose fixed-point interval [excl, excl + W) holds
      // floor(total * u); the elements after it lose its weight.
      const uint64_t t = mulfloor(total, m.uni[j]);
      uint64_t wl = 0;
#pragma unroll
      for (int r = 0; r < kMergeR; ++r)
        if (excl[r] <= t && t - excl[r] < W[r]) {
          wl = W[r];
          rs = r;
        }
      if (rs >= 0) m.pick_w[q] = wl;
      __syncthreads();
      const uint64_t w = m.pick_w[q];
#pragma unroll
      for (int r = 0; r < kMergeR; ++r) {
        if (excl[r] > t) excl[r] -= w;
        if (r == rs) W[r] = 0;
      }
      total -= w;
    } else {
      // No fixed-point mass left: the largest remaining nonzero probability,
      // ties to the lowest flattened position.
      float best = -1.0f;
      int be = 0x7fffffff;
#pragma unroll
      for (int r = 0; r < kMergeR; ++r) {
        if (!((valid >> r) & 1u) || ((taken >> r) & 1u)) continue;
        const float p = __fdiv_rn(ex[r], Sf);
        if (p > 0.0f && p > best) {
          best = p;
          be = tid * kMergeR + r;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
      if (lane == 0) {
        m.fb_p[q][warp] = best;
        m.fb_e[q][warp] = be;
      }
      __syncthreads();
      best = m.fb_p[q][0];
      be = m.fb_e[q][0];
#pragma unroll
      for (int w = 1; w < NW; ++w) {
        const float ob = m.fb_p[q][w];
        const int oe = m.fb_e[q][w];
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
      if (be / kMergeR == tid) rs = be - tid * kMergeR;
    }
    if (rs >= 0) {
      // The pick's outputs from the owner's registers.
#pragma unroll
      for (int r = 0; r < kMergeR; ++r)
        if (r == rs) {
          taken |= 1u << r;
          a.out_picks[j] = (int64_t)b * a.vocab + ki[r];
          a.out_pick_scores[j] = s[r];
        }
    }
  }
  if (tid == 0) {
    *a.out_npicks = n;
    a.out_status[0] = ST_OK;
  }
  return true;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// ------------------------------------------------------------------ the kernel

template <typename TIn, int MODE>
__global__ void __launch_bounds__(NT, 3) row_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>(smem_raw);
  BlockScratch<NT>& bs = sh.bs;
  unsigned char* regA = smem_raw + ((sizeof(Shared) + 127) & ~size_t(127));
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int ES = Elem<TIn>::kSize;
  constexpr int EPU = 16 / ES;
  using IO = UnitIO<TIn>;
  const int S = a.S;
  const int crank = (int)cluster.block_rank();
  const int64_t row = blockIdx.x / S;
  const int tid = threadIdx.x, lane = tid & 31;
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
    for (int c = 0; c < kChunks; ++c) mbar_init(&sh.mbar[c], 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (tid == 0 && has_bulk) {
    unsigned char* dst = reinterpret_cast<unsigned char*>(data) + (b_lo - base16);
    for (int c = 0; c < kChunks; ++c) {
      const uint32_t off = (uint32_t)c * csz;
      if (off >= bulk_bytes) break;
      const uint32_t sz = min(csz, bulk_bytes - off);
      mbar_expect_tx(&sh.mbar[c], sz);
      bulk_g2s(dst + off, reinterpret_cast<const void*>(b_lo + off), sz, &sh.mbar[c]);
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
    local_err |= mark_ids<NT>(reinterpret_cast<const int32_t*>(a.hist) + row * a.hist_stride, hist_length(a, row),
                              V, lo, hi, mask + off_e);
  } else if (a.hist_kind == HIST_IDS64) {
    local_err |= mark_ids<NT>(reinterpret_cast<const int64_t*>(a.hist) + row * a.hist_stride, hist_length(a, row),
                              V, lo, hi, mask + off_e);
  } else if (a.hist_kind == HIST_MASK8 || a.hist_kind == HIST_BITS32) {
    for (int64_t e = tid; e < nel; e += NT) mask[off_e + e] = seen_global(a, row, lo + e);
  }
  __syncthreads();

  // Wait for the bulk chunks (bounded).
  bool timeout = false;
  if (has_bulk) {
    for (int c = 0; c < kChunks; ++c) {
      if ((uint32_t)c * csz >= bulk_bytes) break;
      if (!mbar_wait(&sh.mbar[c], 0)) timeout = true;
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
    const float te = tau_from_groups<NT>(bs, sh.gmax, kGroups, a.kk, T, &sh.err);
    if (tid == 0) sh.tau_eff = te;
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
    tmax = block_max_nan<NT>(bs, tmax);
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
    lsum = block_sum_u64<NT>(bs, lsum);
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
    if (!bad) {
      const float te = tau_from_groups<NT>(bs, sh.gmax, kGroups, a.kk, T, &sh.err);
      if (tid == 0) sh.tau_eff = te;
    } else if (tid == 0) {
      sh.err |= 1 << (M != M ? ST_NAN : (M == NEG ? ST_ALLNEGINF : ST_POSINF));
      sh.tau_eff = __int_as_float(0x7fc00000);
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
        const float tv = temper(v[e], T);
        // A finite score the temperature takes to +inf (T < 1); every element at
        // or above the bound is tested, so the largest ones always are.
        if (tv == __int_as_float(0x7f800000)) atomicOr(remote(cluster, &sh.err, 0), 1 << ST_POSINF);
        if (slot < CAP) {
          rval[slot] = tv;
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
  const int err = sh.err;
  int status = err ? first_err(err) : ST_OK;
  Kept kept = {0, 0.0f, 0};
  int64_t token = -1;
  bool published = false;  // beam: kept list already published by warp 0
  const int n = sh.cand_n;
  // The row maximum is always a candidate when it is finite (tau <= max).
  if (status == ST_OK && n == 0) status = ST_ALLNEGINF;
  if (status == ST_OK) {
    float* sval = reinterpret_cast<float*>(regA);
    int* sidx = reinterpret_cast<int*>(regA + 4 * CAP);
    uint64_t* W = reinterpret_cast<uint64_t*>(regA + 8 * CAP);
    if (!a.force_slow && n <= CAP) {
      float* fv = reinterpret_cast<float*>(W);
      int* fi = reinterpret_cast<int*>(regA + 12 * CAP);
      // Up to 128 candidates: one warp finishes in registers (after the exact
      // prefilter when there are more).
      const float* cv = sh.cand_val;
      const int* ci = sh.cand_idx;
      int m = n;
      if (n > 128) {
        m = prefilter<NT>(bs, sh.cand_val, sh.cand_idx, n, a.kk, fv, fi);
        cv = fv;
        ci = fi;
      }
      if (m <= 128 && MODE == MODE_BEAM) {
        // Warp 0 finishes, publishes the kept list and, in the last leader, merges
        // the beams; the other warps write this beam's kept outputs meanwhile.
        published = true;
        if (tid < 32) {
          kept = m <= 64 ? warp_finish<2>(a, cv, ci, m, uu, &token, kidx, kval)
                         : warp_finish<4>(a, cv, ci, m, uu, &token, kidx, kval);
          if (tid == 0) {
            bs.flag2 = kept.n;
            bs.fval = kept.M;
            bs.u64a = kept.tot;
          }
          named_arrive(1, NT);
          // The lanes' kept-list writes are ordered before lane 0's release.
          __syncwarp();
          BeamWsHeader* hdr = reinterpret_cast<BeamWsHeader*>(a.ws);
          int last = 0;
          if (tid == 0) {
            hdr->status[row] = ST_OK;
            hdr->count[row] = kept.n;
            if (a.out_count) a.out_count[row] = kept.n;
            last = atom_add_acq_rel_gpu(&hdr->counter, 1u) == (unsigned)(a.rows - 1);
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          bool block_merge = false;
          if (last) {
            block_merge = a.force_slow || !beam_merge_warp(a);
            if (tid == 0 && !block_merge) atomicExch(&hdr->counter, 0u);
          }
          if (tid == 0) bs.flag = block_merge;
        } else {
          named_sync(1, NT);
          kept.n = bs.flag2;
          kept.M = bs.fval;
          kept.tot = bs.u64a;
        }
      } else if (m <= 128) {
        if (tid < 32) {
          kept = m <= 64 ? warp_finish<2>(a, cv, ci, m, uu, &token, kidx, kval)
                         : warp_finish<4>(a, cv, ci, m, uu, &token, kidx, kval);
          if (tid == 0) {
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
        kept = leader_fast<NT>(a, bs, fv, fi, m, sval, sidx, W, reinterpret_cast<uint64_t*>(sh.cand_val), kidx, kval);
        if (MODE == MODE_SAMPLE) token = draw_kept<NT>(bs, kidx, kval, kept, uu, reinterpret_cast<uint64_t*>(regA));
      }
      const float Sf = fix_to_float(kept.tot);
      const int first = published ? tid - 32 : tid, stride = published ? NT - 32 : NT;
      for (int j = first < 0 ? kept.n : first; j < kept.n; j += stride) {
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
      // Seen bitmap of the whole row, then the general path.
      uint32_t* bits = reinterpret_cast<uint32_t*>(regA);
      const int nw = (int)((V + 31) >> 5);
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
      auto seen = [&](int64_t i) -> bool { return (bits[i >> 5] >> (i & 31)) & 1u; };
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
      unsigned char* scratch = regA + (((size_t)nw * 4 + 127) & ~size_t(127));
      kept = leader_slow<NT, TIn, MODE>(a, bs, scratch, row, bM, bL, uu, &token, seen, emit);
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
  if (published) {
    __syncthreads();  // warp 0's merge attempt is done
    if (!bs.flag) return;
    if (a.force_slow || !beam_merge_block(a)) beam_merge(a, sh, regA);
    __syncthreads();
    if (tid == 0) atomicExch(&hdr->counter, 0u);
    return;
  }
  if (tid == 0) {
    hdr->status[row] = status;
    hdr->count[row] = kept.n;
    if (a.out_count) a.out_count[row] = kept.n;
  }
  // The barrier orders the block's kept-list writes before thread 0's atomic,
  // whose release publishes them and whose acquire (in the last leader) orders
  // the other leaders' lists before the merge's reads.
  __syncthreads();
  if (tid == 0) bs.flag = atom_add_acq_rel_gpu(&hdr->counter, 1u) == (unsigned)(a.rows - 1);
  __syncthreads();
  if (!bs.flag) return;
  if (tid < 32) {
    const bool done = !a.force_slow && beam_merge_warp(a);
    if (tid == 0) bs.flag2 = done;
  }
  __syncthreads();
  if (!bs.flag2 && (a.force_slow || !beam_merge_block(a))) beam_merge(a, sh, regA);
  __syncthreads();
  if (tid == 0) atomicExch(&hdr->counter, 0u);
}

// The beam merge alone, over kept lists already in a workspace (the vocab-sharded
// beam step): one CTA, the same cascade as the row kernel's last leader.
__global__ void __launch_bounds__(NT) beam_merge_kernel(const RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>(smem_raw);
  unsigned char* regA = smem_raw + ((sizeof(Shared) + 127) & ~size_t(127));
  const int tid = threadIdx.x;
  if (tid < 32) {
    const bool done = !a.force_slow && beam_merge_warp(a);
    if (tid == 0) sh.bs.flag2 = done;
  }
  __syncthreads();
  if (!sh.bs.flag2 && (a.force_slow || !beam_merge_block(a))) beam_merge(a, sh, regA);
}

// ---------------------------------------------------------------- host launch

template <typename TIn, int MODE>
cudaError_t launch_t(const RowArgs& a, size_t smem, cudaStream_t stream) {
  auto kern = row_kernel<TIn, MODE>;
  static int configured[64] = {0};
  static int max_dyn[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
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

}  // namespace

size_t shared_static_bytes() { return (sizeof(Shared) + 127) & ~size_t(127); }

// The merge's shared-memory staging (scores, weights and flattened ids of up to
// 1024 entries) after the Shared block.
constexpr size_t kMergeRegion = 16384;

cudaError_t launch_beam_merge(const RowArgs& a, cudaStream_t stream) {
  beam_merge_kernel<<<1, NT, shared_static_bytes() + kMergeRegion, stream>>>(a);
  return cudaGetLastError();
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
