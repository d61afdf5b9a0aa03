// sv_loop_guard.cu -- batched loop guard (runtime_shared.py:156-167, _repeating).
//
// Verdict for a row of L tokens: L >= window*repeats and the last `window` tokens
// occur at least `repeats` times (overlapping starts allowed, the tail itself
// counted).
//
// Rows with a stride are streamed: every window start's first token is compared
// with the tail's first token, the reference's own filter (:163), over 16-byte
// vector loads (all of a thread's loads of a pass in flight at once), and the few
// candidates are then verified against the whole tail, one warp per candidate,
// from L2.  The work per row is one compare per token plus the verifications, so
// the kernel runs at the speed of the loads.  A row of at most one pass (16384
// int32 tokens) is one 1024-thread CTA (loop_guard_row_kernel); longer rows are
// split across a cluster of up to 8 CTAs whose counts meet in rank 0 through
// distributed shared memory (loop_guard_scan_kernel).
//
// With row stride 0 (rows given by lengths only) loop_guard_kernel takes the rows:
// one CTA per row.  Tokens are staged chunk by chunk in shared memory;
// each thread owns a contiguous run of window starts and rolls a polynomial hash
// (mod 2^32, odd base, over a 32-bit mix of each token) along it; a start whose
// hash equals the tail's hash is verified token by token, so the verdict is exact
// (a hash collision costs one verification, never a wrong verdict).  The scan stops once
// `repeats` occurrences are found.  A chunk holds 16640 starts, so a 16K-token row
// is staged once (16-byte vectors when the row is aligned); the rolling step
// h(s+1) = h(s) B + (x[s+w] - x[s] B^w) keeps one multiply on the dependency chain.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/starvector_sampling.h"
#include "sv_guard.cuh"
#include "sv_internal.h"

namespace sv {

constexpr int LG_NT = 256;
constexpr int LG_PER = 65;                  // starts per thread (odd: no bank conflicts)
constexpr int LG_CH = LG_NT * LG_PER;       // starts per chunk (a 16K-token row in one)
constexpr int LG_MAXW = 1024;               // window limit
constexpr uint32_t LG_BASE = 0x9E3779B1u;

// A token as 32 bits for the hash (an int64 token folds its high half in).
__device__ __forceinline__ uint32_t tok32(int32_t x) { return (uint32_t)x; }
__device__ __forceinline__ uint32_t tok32(int64_t x) { return (uint32_t)x ^ ((uint32_t)(x >> 32) * 0x85EBCA6Bu); }

// The window hash sum_j p[j] B^(w-1-j) (mod 2^32) as four interleaved Horner
// chains (j = k mod 4, step B^4), so its latency is a quarter of one chain's.
template <typename Tok>
__device__ __forceinline__ uint32_t hash_window(const Tok* p, int w) {
  constexpr uint32_t B2 = LG_BASE * LG_BASE, B3 = B2 * LG_BASE, B4 = B2 * B2;
  uint32_t h[4] = {0, 0, 0, 0};
  int j = 0;
  for (; j + 4 <= w; j += 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = h[k] * B4 + tok32(p[j + k]);
  }
  // Chain k holds p[k], p[k+4], ..., p[k+4(n-1)] with weights B^(4(n-1-i)); the
  // window weights p[4i+k] by B^(4(n-1-i) + 3-k) for its first 4n tokens.
  uint32_t r = h[0] * B3 + h[1] * B2 + h[2] * LG_BASE + h[3];
  for (; j < w; ++j) r = r * LG_BASE + tok32(p[j]);
  return r;
}

template <typename Tok>
__global__ void __launch_bounds__(LG_NT) loop_guard_kernel(const Tok* __restrict__ tokens, int64_t stride,
                                                           const int32_t* __restrict__ lengths, int window,
                                                           int repeats, uint8_t* __restrict__ verdict) {
  extern __shared__ __align__(16) unsigned char lg_smem[];
  Tok* buf = reinterpret_cast<Tok*>(lg_smem);                       // LG_CH + window - 1
  Tok* tail = buf + LG_CH + LG_MAXW;                                 // window
  __shared__ int count;
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  int64_t L = lengths[row];
  if (stride > 0 && L > stride) L = stride;  // a row holds at most `stride` tokens
  const Tok* t = tokens + row * stride;
  if (L < (int64_t)window * repeats) {
    if (tid == 0) verdict[row] = 0;
    return;
  }
  for (int j = tid; j < window; j += LG_NT) tail[j] = t[L - window + j];
  if (tid == 0) count = 0;
  // B^w: the rolling step h(s+1) = h(s) B + x[s+w] - x[s] B^w.
  uint32_t bw = 1, bq = LG_BASE;
  for (int e = window; e; e >>= 1, bq *= bq)
    if (e & 1) bw *= bq;
  // 16-byte vectors where the row allows them.
  constexpr int VE = 16 / (int)sizeof(Tok);
  const bool vec = (reinterpret_cast<uintptr_t>(t) & 15) == 0;
  const int64_t nstarts = L - window + 1;
  uint32_t ht = 0;
  for (int64_t c0 = 0; c0 < nstarts; c0 += LG_CH) {
    const int64_t cn = nstarts - c0 < LG_CH ? nstarts - c0 : LG_CH;
    const int64_t ntok = cn + window - 1;
    const Tok* src = t + c0;
    if (vec) {
      const int64_t nv = ntok / VE;
      for (int64_t q = tid; q < nv; q += LG_NT)
        reinterpret_cast<uint4*>(buf)[q] = reinterpret_cast<const uint4*>(src)[q];
      for (int64_t j = nv * VE + tid; j < ntok; j += LG_NT) buf[j] = src[j];
    } else {
      for (int64_t j = tid; j < ntok; j += LG_NT) buf[j] = src[j];
    }
    __syncthreads();
    if (c0 == 0) ht = hash_window(tail, window);  // every thread, from shared memory
    const int s0 = tid * LG_PER;
    if (s0 < cn) {
      uint32_t h = hash_window(buf + s0, window);
      const int s1 = s0 + LG_PER < cn ? s0 + LG_PER : (int)cn;
      for (int s = s0; s < s1; ++s) {
        if (h == ht) {
          bool eq = true;
          for (int j = 0; j < window && eq; ++j) eq = buf[s + j] == tail[j];
          if (eq) atomicAdd(&count, 1);
        }
        if (s + 1 < s1)
          h = h * LG_BASE + (tok32(buf[s + window]) - tok32(buf[s]) * bw);
      }
    }
    __syncthreads();
    if (count >= repeats) break;
  }
  if (tid == 0) verdict[row] = count >= repeats;
}

size_t loop_guard_smem(int token_bytes) { return (size_t)(LG_CH + 2 * LG_MAXW) * token_bytes; }

namespace cg = cooperative_groups;

constexpr int LS_NT = 256;
constexpr int LS_U = 4;  // 16-byte vectors per thread per pass

__device__ __forceinline__ void lg_cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }
__device__ __forceinline__ void lg_cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <typename Tok, int P>
__global__ void __cluster_dims__(P, 1, 1) __launch_bounds__(LS_NT, sizeof(Tok) == 4 ? 7 : 6)
    loop_guard_scan_kernel(const Tok* __restrict__ tokens, int64_t stride, const int32_t* __restrict__ lengths,
                           int w, int repeats, uint8_t* __restrict__ verdict) {
  constexpr int VE = 16 / (int)sizeof(Tok);
  constexpr int PASS = LS_NT * LS_U * VE;  // window starts per pass
  constexpr int NWARP = LS_NT / 32;
  constexpr unsigned FULL = 0xffffffffu;
  __shared__ Tok tail[LG_MAXW];
  __shared__ int cand[PASS];
  __shared__ int ncand, count, total;  // total: the cluster's count, in rank 0
  cg::cluster_group cl = cg::this_cluster();
  const int part = (int)cl.block_rank();
  const int64_t row = blockIdx.x / P;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const Tok* t = tokens + row * stride;
  // This CTA's share of the row's possible window starts, from the stride (so the
  // first loads need not wait for the length): [a, a + per), a a multiple of VE so
  // that vectors begin on a start.  Loads stay inside the row's stride.
  const int S = (int)stride;  // < 2^30 (host check): 32-bit positions
  const int smax = S - w + 1 > 0 ? S - w + 1 : 0;
  const int per = ((smax + P - 1) / P + VE - 1) / VE * VE;
  const int a = part * per;
  const bool vec = (reinterpret_cast<uintptr_t>(t) & 15) == 0;
  Tok v[LS_U][VE];
  auto load_pass = [&](int p0, int lim) {
#pragma unroll
    for (int u = 0; u < LS_U; ++u) {
      const int pos = p0 + (u * LS_NT + tid) * VE;
      if (vec && pos + VE <= lim) {
        const uint4 q = *reinterpret_cast<const uint4*>(t + pos);
        memcpy(&v[u][0], &q, 16);
      } else {
#pragma unroll
        for (int j = 0; j < VE; ++j) v[u][j] = pos + j < lim ? t[pos + j] : Tok(0);
      }
    }
  };
  if (tid == 0) {
    ncand = 0;
    count = 0;
    total = 0;
  }
  if (a < smax) load_pass(a, S);
  int L = lengths[row];
  // The tail of a full row (the common case), beside the first loads.
  if (S >= w)
    for (int k = tid; k < w; k += LS_NT) tail[k] = t[S - w + k];
  lg_cluster_arrive();  // rank 0's `total` is zero before any CTA adds to it
  __syncthreads();
  if (L > S) L = S;
  if ((int64_t)L < (int64_t)w * repeats) {  // the same for every CTA of the cluster: none waits
    if (part == 0 && tid == 0) verdict[row] = 0;
    return;
  }
  if (L != S) {
    for (int k = tid; k < w; k += LS_NT) tail[k] = t[L - w + k];
    __syncthreads();
  }
  const int nst = L - w + 1;  // window starts
  const int b = a + per < nst ? a + per : nst;
  const Tok t0 = tail[0];
  for (int p0 = a; p0 < b; p0 += PASS) {
#pragma unroll
    for (int u = 0; u < LS_U; ++u) {
      const int pos = p0 + (u * LS_NT + tid) * VE;
#pragma unroll
      for (int j = 0; j < VE; ++j)
        if (v[u][j] == t0 && pos + j < b) cand[atomicAdd(&ncand, 1)] = pos + j - p0;
    }
    __syncthreads();
    const int nc = ncand;
    if (p0 + PASS < b) load_pass(p0 + PASS, L);  // the next pass's loads fly during the checks
    for (int c = warp; c < nc; c += NWARP) {
      int done = lane == 0 ? *reinterpret_cast<volatile int*>(&count) >= repeats : 0;
      if (__shfl_sync(FULL, done, 0)) break;
      const int st = p0 + cand[c];
      bool eq = true;
      for (int k = lane; k < w && eq; k += 32) eq = t[st + k] == tail[k];
      if (__all_sync(FULL, eq) && lane == 0) atomicAdd(&count, 1);
    }
    __syncthreads();
    if (count >= repeats || p0 + PASS >= b) break;  // read after the barrier: the same in every thread
    if (tid == 0) ncand = 0;
    __syncthreads();
  }
  lg_cluster_wait();  // every CTA has initialised its `total`
  if (tid == 0 && count) atomicAdd(cl.map_shared_rank(&total, 0), count);
  lg_cluster_arrive();  // the adds are done (release) ...
  lg_cluster_wait();    // ... before rank 0 reads, and rank 0's memory outlives them
  if (part == 0 && tid == 0) verdict[row] = total >= repeats;
}


constexpr int LR_NT = 1024;

// Rows of at most one pass (a 16384-token int32 row, 8192 int64): one CTA of 1024
// threads per row, the whole row's loads in flight at once, no cluster, one block
// barrier.  Each warp keeps its own candidates (at most one per position it loaded)
// in its region of dynamic shared memory and checks them itself.
template <typename Tok>
__global__ void __launch_bounds__(LR_NT, 2)
    loop_guard_row_kernel(const Tok* __restrict__ tokens, int64_t stride, const int32_t* __restrict__ lengths,
                          int w, int repeats, uint8_t* __restrict__ verdict) {
  constexpr int VE = 16 / (int)sizeof(Tok);
  constexpr int NWARP = LR_NT / 32;
  constexpr int WCAP = 32 * LS_U * VE;  // positions a warp covers: its candidates' room
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ int cand[];
  __shared__ int wcount[NWARP];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const Tok* t = tokens + row * stride;
  const int S = (int)stride;
  const bool vec = (reinterpret_cast<uintptr_t>(t) & 15) == 0;
  Tok v[LS_U][VE];
#pragma unroll
  for (int u = 0; u < LS_U; ++u) {
    const int pos = (u * LR_NT + tid) * VE;
    if (vec && pos + VE <= S) {
      const uint4 q = *reinterpret_cast<const uint4*>(t + pos);
      memcpy(&v[u][0], &q, 16);
    } else {
#pragma unroll
      for (int j = 0; j < VE; ++j) v[u][j] = pos + j < S ? t[pos + j] : Tok(0);
    }
  }
  int L = lengths[row];
  Tok t0 = S >= w ? t[S - w] : Tok(0);  // the tail's first token of a full row, beside the loads
  if (L > S) L = S;
  if ((int64_t)L < (int64_t)w * repeats) {
    if (tid == 0) verdict[row] = 0;
    return;
  }
  if (L != S) t0 = t[L - w];
  const int nst = L - w + 1;
  // Each warp's candidates (its own region; ballots, no block atomics), checked by
  // the warp itself against the tail read from L2.
  int* wc = cand + warp * WCAP;
  int nc = 0;
#pragma unroll
  for (int u = 0; u < LS_U; ++u) {
    const int pos = (u * LR_NT + tid) * VE;
#pragma unroll
    for (int j = 0; j < VE; ++j) {
      const bool hit = v[u][j] == t0 && pos + j < nst;
      const unsigned bal = __ballot_sync(FULL, hit);
      if (hit) wc[nc + __popc(bal & ((1u << lane) - 1u))] = pos + j;
      nc += __popc(bal);
    }
  }
  __syncwarp();
  int count = 0;
  const Tok* tail = t + (L - w);
  for (int c = 0; c < nc && count < repeats; ++c) {
    const int st = wc[c];
    bool eq = true;
    for (int k = lane; k < w && eq; k += 32) eq = t[st + k] == tail[k];
    count += __all_sync(FULL, eq);
  }
  if (lane == 0) wcount[warp] = count;
  __syncthreads();
  if (tid == 0) {
    int total = 0;
#pragma unroll
    for (int k = 0; k < NWARP; ++k) total += wcount[k];
    verdict[row] = total >= repeats;
  }
}

template <typename Tok>
cudaError_t launch_scan(const Tok* tokens, int rows, int64_t stride, const int32_t* lengths, int window, int repeats,
                        uint8_t* verdict, cudaStream_t stream) {
  constexpr int RPASS = LR_NT * LS_U * (16 / (int)sizeof(Tok));
  if (stride <= RPASS) {
    const size_t smem = (size_t)RPASS * sizeof(int);
    static int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaFuncSetAttribute(loop_guard_row_kernel<Tok>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured[dev] = 1;
    }
    loop_guard_row_kernel<Tok><<<rows, LR_NT, smem, stream>>>(tokens, stride, lengths, window, repeats, verdict);
    return cudaGetLastError();
  }
  // CTAs per row: about one pass of window starts each, at most 8 (a portable cluster).
  constexpr int PASS = LS_NT * LS_U * (16 / (int)sizeof(Tok));
  const int64_t want = (stride + PASS - 1) / PASS;
  const int P = want >= 8 ? 8 : want >= 4 ? 4 : want >= 2 ? 2 : 1;
  const dim3 grid((unsigned)((int64_t)rows * P));
  switch (P) {
    case 1: loop_guard_scan_kernel<Tok, 1><<<grid, LS_NT, 0, stream>>>(tokens, stride, lengths, window, repeats, verdict); break;
    case 2: loop_guard_scan_kernel<Tok, 2><<<grid, LS_NT, 0, stream>>>(tokens, stride, lengths, window, repeats, verdict); break;
    case 4: loop_guard_scan_kernel<Tok, 4><<<grid, LS_NT, 0, stream>>>(tokens, stride, lengths, window, repeats, verdict); break;
    default: loop_guard_scan_kernel<Tok, 8><<<grid, LS_NT, 0, stream>>>(tokens, stride, lengths, window, repeats, verdict); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_loop_guard(const void* tokens, int token_bytes, int rows, int64_t stride, const int32_t* lengths,
                              int window, int repeats, uint8_t* verdict, cudaStream_t stream) {
  if (stride > 0 && stride < (int64_t)1 << 30) {
    if (token_bytes == 4)
      return launch_scan(reinterpret_cast<const int32_t*>(tokens), rows, stride, lengths, window, repeats, verdict,
                         stream);
    return launch_scan(reinterpret_cast<const int64_t*>(tokens), rows, stride, lengths, window, repeats, verdict,
                       stream);
  }
  const size_t smem = loop_guard_smem(token_bytes);
  int dev = 0;
  cudaGetDevice(&dev);
  static int configured[64][2] = {};
  const bool fresh = dev >= 0 && dev < 64 && !configured[dev][token_bytes == 8];
  if (token_bytes == 4) {
    if (fresh) {
      cudaFuncSetAttribute(loop_guard_kernel<int32_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured[dev][0] = 1;
    }
    loop_guard_kernel<int32_t><<<rows, LG_NT, smem, stream>>>(reinterpret_cast<const int32_t*>(tokens), stride,
                                                                lengths, window, repeats, verdict);
  } else {
    if (fresh) {
      cudaFuncSetAttribute(loop_guard_kernel<int64_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured[dev][1] = 1;
    }
    loop_guard_kernel<int64_t><<<rows, LG_NT, smem, stream>>>(reinterpret_cast<const int64_t*>(tokens), stride,
                                                                lengths, window, repeats, verdict);
  }
  return cudaGetLastError();
}

int loop_guard_max_window() { return LG_MAXW; }

// ---------------------------------------------------------------------------
// Incremental loop guard: one sequence's verdict from its window-occurrence table
// (sv_guard.cuh) in time independent of the sequence's length.  A check enters
// the windows ending at positions [from, L) and probes the table for the tail.
// The latency of a check is a handful of dependent L2 round trips, so each step
// keeps them few: up to GI_DIRECT new windows (a decode loop enters 16 per check)
// are staged with the tail in shared memory by one coalesced load and hashed
// eight lanes per window, all windows at once (each lane sums tok * B^(w-1-k) over
// its positions k, three shuffles add the group's sums: the hash is a sum mod 2^32,
// so the order does not matter), then entered together.  More windows (a table
// built in one call) are hashed by contiguous runs per thread, the first window
// directly and the rest rolled.  The tail's occurrences are counted until
// `repeats` distinct starts match (the tail itself among them, as the reference
// counts it): among this call's windows straight from shared memory, among the
// older ones through the table's probe chain, read 32 slots per load, each hash
// match verified token by token (the tail's own entry counts without a check).

constexpr int GI_NT = 160;  // warp 0 counts while four warps enter 16 windows per pass
constexpr int GI_DIRECT = 256;

__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename Tok>
__global__ void __launch_bounds__(GI_NT) guard_incremental_kernel(unsigned long long* table, int64_t mask,
                                                                  const Tok* __restrict__ tokens, int64_t from,
                                                                  int64_t L, int w, int repeats, uint8_t* verdict,
                                                                  int32_t* status) {
  __shared__ Tok stage[GI_DIRECT + LG_MAXW];
  __shared__ uint32_t pw[LG_MAXW];  // B^(w-1-k)
  __shared__ int full;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARP = GI_NT / 32;
  if (L < w) {  // no whole window yet
    if (tid == 0) {
      *verdict = 0;
      if (status) *status = SV_ST_OK;
    }
    return;
  }
  if (tid == 0) full = 0;
  const int64_t e0 = from > (int64_t)w - 1 ? from : (int64_t)w - 1;
  const int64_t n = L > e0 ? L - e0 : 0;  // windows to enter
  const bool direct = n <= GI_DIRECT;
  // Staged tokens: the windows to enter (direct) and always the tail.
  const int64_t s0 = (direct && n ? e0 : L - 1) - w + 1;
  const int slen = (int)(L - s0);
  for (int j = tid; j < slen; j += GI_NT) stage[j] = tokens[s0 + j];
  for (int k = tid; k < w; k += GI_NT) pw[k] = guard_pow(kGuardBase, w - 1 - k);
  __syncthreads();
  const Tok* tail = stage + (slen - w);
  const bool judged = L >= (int64_t)w * repeats;
  // Warp 0's count of the tail's occurrences among the windows whose start lies
  // below `upto`, from the table: it reads the tail hash's probe chain 32 slots per
  // load and verifies each hash match token by token (the tail's own entry counts
  // without a check).
  auto probe = [&](int64_t upto, int count) {
    uint32_t ht = 0;
    for (int k = lane; k < w; k += 32) ht += guard_tok(tail[k]) * pw[k];
    ht = warp_sum_u32(ht);
    const uint32_t self = (uint32_t)(L - w);
    const int64_t slot0 = guard_mix(ht) & mask;
    for (int64_t i0 = 0; i0 <= mask && count < repeats; i0 += 32) {
      const unsigned long long e = i0 + lane <= mask ? table[(slot0 + i0 + lane) & mask] : kGuardEmpty;
      const unsigned empty = __ballot_sync(0xffffffffu, e == kGuardEmpty);
      const unsigned before = empty ? (1u << (__ffs(empty) - 1)) - 1u : 0xffffffffu;  // the chain's slots
      unsigned cand = __ballot_sync(0xffffffffu, (uint32_t)(e >> 32) == ht) & before;
      while (cand && count < repeats) {
        const int c = __ffs(cand) - 1;
        cand &= cand - 1;
        const int64_t st = __shfl_sync(0xffffffffu, (unsigned)(e & 0xffffffffu), c);
        if (st >= upto) continue;  // one of this call's windows: counted from shared memory
        if (st == self) {
          ++count;
          continue;
        }
        bool eq = st + w <= L;
        for (int k = lane; k < w && eq; k += 32) eq = tokens[st + k] == tail[k];
        if (__all_sync(0xffffffffu, eq)) ++count;
      }
      if (empty) break;
    }
    return count;
  };
  int count = 0;
  if (direct) {
    // Warps 1.. enter this call's windows (eight lanes per window, 16 per pass; the
    // loop test is warp-uniform) while warp 0 counts the tail among them straight
    // from shared memory and probes the table for the older windows only, so the
    // probe does not wait for the inserts.
    const int64_t first_new = n ? e0 - w + 1 : L - w + 1;
    if (warp > 0) {
      const int g = lane >> 3, gl = lane & 7;
      for (int64_t e = e0 + (warp - 1) * 4 + g; e - g < L; e += (NWARP - 1) * 4) {
        const bool act = e < L;
        uint32_t h = 0;
        if (act) {
          const int o = (int)(e - w + 1 - s0);
          for (int k = gl; k < w; k += 8) h += guard_tok(stage[o + k]) * pw[k];
        }
#pragma unroll
        for (int m = 4; m; m >>= 1) h += __shfl_xor_sync(0xffffffffu, h, m);
        if (act && gl == 0 && !guard_insert(table, mask, h, (uint32_t)(e - w + 1))) full = 1;
      }
    } else if (judged) {
      // This call's windows hashed four at a time (eight lanes each) against the
      // tail's hash; a match is verified token by token in shared memory.
      uint32_t ht = 0;
      for (int k = lane; k < w; k += 32) ht += guard_tok(tail[k]) * pw[k];
      ht = warp_sum_u32(ht);
      const int g = lane >> 3, gl = lane & 7;
      for (int64_t st0 = first_new; st0 <= L - w && count < repeats; st0 += 4) {
        const int64_t st = st0 + g;
        const bool act = st <= L - w;
        uint32_t h = 0;
        if (act) {
          const int o = (int)(st - s0);
          for (int k = gl; k < w; k += 8) h += guard_tok(stage[o + k]) * pw[k];
        }
#pragma unroll
        for (int m = 4; m; m >>= 1) h += __shfl_xor_sync(0xffffffffu, h, m);
        unsigned hit = __ballot_sync(0xffffffffu, act && gl == 0 && h == ht);
        while (hit && count < repeats) {
          const int c = __ffs(hit) - 1;
          hit &= hit - 1;
          const int o = (int)(st0 + (c >> 3) - s0);
          bool eq = true;
          for (int k = lane; k < w && eq; k += 32) eq = stage[o + k] == tail[k];
          count += __all_sync(0xffffffffu, eq);
        }
      }
      if (count < repeats) count = probe(first_new, count);
    }
    __syncthreads();  // every insert has finished (the status)
  } else {
    const uint32_t bw = guard_pow(kGuardBase, w);
    const int64_t per = (n + GI_NT - 1) / GI_NT;
    const int64_t a = e0 + tid * per, b = a + per < L ? a + per : L;
    if (a < b) {
      uint32_t h = 0;
      for (int k = 0; k < w; ++k) h = h * kGuardBase + guard_tok(tokens[a - w + 1 + k]);
      for (int64_t e = a; e < b; ++e) {
        if (!guard_insert(table, mask, h, (uint32_t)(e - w + 1))) full = 1;
        if (e + 1 < b) h = h * kGuardBase + guard_tok(tokens[e + 1]) - guard_tok(tokens[e + 1 - w]) * bw;
      }
    }
    __syncthreads();
    if (warp == 0 && judged) count = probe(L - w + 1, 0);
  }
  if (tid == 0) {
    *verdict = count >= repeats;
    if (status) *status = full ? SV_ST_GUARD_FULL : SV_ST_OK;
  }
}

}  // namespace sv

// See include/starvector_sampling.h.
extern "C" int sv_loop_guard_incremental(unsigned long long* table, int64_t table_entries, const void* tokens,
                                         int32_t token_bytes, int64_t insert_from, int64_t length, int32_t window,
                                         int32_t repeats, uint8_t* out_verdict, int32_t* out_status, void* stream) {
  using namespace sv;
  if (!table || !tokens || !out_verdict) return SV_E_ARG;
  if (token_bytes != 4 && token_bytes != 8) return SV_E_DTYPE;
  if (table_entries < 2 || (table_entries & (table_entries - 1))) return SV_E_SHAPE;
  if (length < 0 || insert_from < 0 || insert_from > length || length > 0x7fffffffLL) return SV_E_SHAPE;
  if (window < 1 || window > LG_MAXW || repeats < 1) return SV_E_RANGE;
  if (reinterpret_cast<uintptr_t>(tokens) % token_bytes || reinterpret_cast<uintptr_t>(table) % 8) return SV_E_ALIGN;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (token_bytes == 4)
    guard_incremental_kernel<int32_t><<<1, GI_NT, 0, st>>>(table, table_entries - 1,
                                                           static_cast<const int32_t*>(tokens), insert_from, length,
                                                           window, repeats, out_verdict, out_status);
  else
    guard_incremental_kernel<int64_t><<<1, GI_NT, 0, st>>>(table, table_entries - 1,
                                                           static_cast<const int64_t*>(tokens), insert_from, length,
                                                           window, repeats, out_verdict, out_status);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}
