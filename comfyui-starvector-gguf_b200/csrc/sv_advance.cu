// sv_advance.cu -- the beam loop's per-step decision on the device
// (runtime_shared.py:237-259), so that the loop needs no host round trip per token.
//
// After sv_beam_step has drawn the step's picks (beam * V + token) and their
// scores, the reference decides on the host which candidates continue:
//   hits[j]   = last step or _ends(running[parent_j] + [token_j])       (:240-241)
//   live[j]   = picked[j] - 1e9 * hits[j]                     (doubles, :245)
//   order     = the first `beams` indices of live sorted descending, stably (:246)
//   running_scores = live[order] + [-1e9] * (beams - len(order)), given to the next
//               step as float32 (torch.tensor of Python floats, :231)      (:247)
//   order    += [order[0]] * (beams - len(order))                           (:248)
//   seen      = seen[parents[order]]; seen[b, tokens[order][b]] = True      (:258-259)
// One launch does all of it.  Every block recomputes the (at most 64-pick)
// decision in shared memory, then copies its share of the seen bitmaps; block 0
// writes the decision.  _ends needs only each running row's last len(stop_ids)
// tokens, kept on the device as a tail per row and advanced here; the rows' whole
// token histories (for the loop guard on running[0], :254) are optionally carried
// along the same way, and so is each row's rolling window hash, whose window
// ending at this step goes into the incremental loop guard's occurrence table.  The finished
// list, the stop tests and the loop guard stay on the host, which replays the
// reference's bookkeeping from the steps' records once per block of steps and
// checks the device's parents and tokens against its own.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/starvector_sampling.h"
#include "sv_guard.cuh"

namespace {

constexpr int ANT = 256;
constexpr int kMaxPicks = 64;
constexpr int kMaxStop = 16;

struct AdvanceArgs {
  const int64_t* picks;
  const float* pick_scores;
  const int32_t* n_picks;
  const int32_t* status;
  int beams, num_picks, n_stop;
  int64_t vocab;
  int step, last;
  const int64_t* stop_ids;
  int64_t eos_id;
  const int64_t* tails_in;
  int64_t* tails_out;
  float* running_out;
  int64_t* parents_out;
  int64_t* tokens_out;
  const uint32_t* seen_in;
  uint32_t* seen_out;
  int64_t seen_words, seen_stride;
  const int32_t* hist_in;
  int32_t* hist_out;
  int64_t hist_stride;
  const uint32_t* whash_in;
  uint32_t* whash_out;
  unsigned long long* guard_table;
  int64_t guard_mask;
  int window;
};

__global__ void __launch_bounds__(ANT) beam_advance_kernel(const AdvanceArgs a) {
  __shared__ int64_t par[kMaxPicks], tok[kMaxPicks];
  __shared__ double live[kMaxPicks];
  __shared__ int order[kMaxPicks];
  __shared__ int64_t stop[kMaxStop];
  __shared__ int ok_s, m_s, n_s;
  const int tid = threadIdx.x;
  if (tid < a.n_stop) stop[tid] = a.stop_ids[tid];
  if (tid == 0) {
    const int n = *a.n_picks;
    ok_s = *a.status == 0 && n >= 1 && n <= a.num_picks;
    n_s = n;
  }
  __syncthreads();
  int n = ok_s ? n_s : 0;
  if (tid < n) {
    const int64_t pick = a.picks[tid];
    const int64_t p = pick / a.vocab, t = pick - p * a.vocab;
    par[tid] = p;
    tok[tid] = t;
    if (pick < 0 || p >= a.beams || a.pick_scores[tid] != a.pick_scores[tid]) ok_s = 0;  // not a valid draw
  }
  __syncthreads();
  const int ok = ok_s;
  n = ok ? n : 0;
  if (tid == 0) m_s = n < a.beams ? n : a.beams;
  if (tid < n) {
    const int64_t p = par[tid], t = tok[tid];
    bool hit = a.last || t == a.eos_id;
    if (!hit && a.n_stop > 0 && a.step + 1 >= a.n_stop && t == stop[a.n_stop - 1]) {
      // The candidate's last n_stop tokens: the parent's tail without its oldest
      // entry, then t.
      bool same = true;
      for (int k = 0; k + 1 < a.n_stop; ++k) same &= a.tails_in[p * a.n_stop + k + 1] == stop[k];
      hit = same;
    }
    live[tid] = (double)a.pick_scores[tid] - (hit ? 1e9 : 0.0);
  }
  __syncthreads();
  if (tid < n) {
    // Stable descending rank: larger values first, equal values in pick order.
    const double v = live[tid];
    int rank = 0;
    for (int i = 0; i < n; ++i) rank += live[i] > v || (live[i] == v && i < tid);
    if (rank < a.beams) order[rank] = tid;
  }
  __syncthreads();
  const int m = m_s;
  if (blockIdx.x == 0 && tid < a.beams) {
    const int r = tid;
    if (ok) {
      const int j = r < m ? order[r] : order[0];
      const int64_t p = par[j], t = tok[j];
      a.running_out[r] = r < m ? (float)live[j] : (float)-1e9;
      a.parents_out[r] = p;
      a.tokens_out[r] = t;
      for (int k = 0; k < a.n_stop; ++k)
        a.tails_out[r * a.n_stop + k] = k + 1 < a.n_stop ? a.tails_in[p * a.n_stop + k + 1] : t;
      if (a.guard_table) {
        // The row's window ending at this step, rolled from its parent's, and its
        // entry in the loop guard's occurrence table (sv_guard.cuh).
        uint32_t h = a.whash_in[p] * sv::kGuardBase + sv::guard_tok((int32_t)t);
        if (a.step >= a.window)
          h -= sv::guard_tok(a.hist_in[p * a.hist_stride + a.step - a.window]) * sv::guard_pow(sv::kGuardBase, a.window);
        a.whash_out[r] = h;
        if (a.step >= a.window - 1) sv::guard_insert(a.guard_table, a.guard_mask, h, (uint32_t)(a.step - a.window + 1));
      }
    } else {
      // A failed step (the host raises when it reads the record): every row keeps
      // its own state, the running scores restart as at the first step and the
      // decoder is fed token 0.
      a.running_out[r] = r == 0 ? 0.f : (float)-1e9;
      a.parents_out[r] = r;
      a.tokens_out[r] = 0;
      for (int k = 0; k < a.n_stop; ++k) a.tails_out[r * a.n_stop + k] = a.tails_in[r * a.n_stop + k];
      if (a.guard_table) a.whash_out[r] = a.whash_in[r];
    }
  }
  // The rows' state, out of place: seen_out[b] = seen_in[parent_b] with the bit of
  // token_b set; hist_out[b] = hist_in[parent_b][0, step) followed by token_b.
  const int64_t seen_total = a.seen_out ? (int64_t)a.beams * a.seen_words : 0;
  const int64_t hist_row = a.step + 1;
  const int64_t total = seen_total + (a.hist_out ? (int64_t)a.beams * hist_row : 0);
  for (int64_t k = (int64_t)blockIdx.x * ANT + tid; k < total; k += (int64_t)gridDim.x * ANT) {
    const bool is_seen = k < seen_total;
    const int64_t kk = is_seen ? k : k - seen_total;
    const int64_t width = is_seen ? a.seen_words : hist_row;
    const int b = (int)(kk / width);
    const int64_t w = kk - (int64_t)b * width;
    int64_t p = b, t = -1;
    if (ok) {
      const int j = b < m ? order[b] : order[0];
      p = par[j];
      t = tok[j];
    }
    if (is_seen) {
      uint32_t v = a.seen_in[p * a.seen_stride + w];
      if (t >= 0 && (t >> 5) == w) v |= 1u << (t & 31);
      a.seen_out[b * a.seen_stride + w] = v;
    } else {
      a.hist_out[b * a.hist_stride + w] = w < a.step ? a.hist_in[p * a.hist_stride + w] : (int32_t)(t < 0 ? 0 : t);
    }
  }
}

}  // namespace

// See include/starvector_sampling.h.
extern "C" int sv_beam_advance(const int64_t* picks, const float* pick_scores, const int32_t* n_picks,
                               const int32_t* status, int32_t beams, int32_t vocab, int32_t num_picks, int32_t step,
                               int32_t last, const int64_t* stop_ids, int32_t n_stop, int64_t eos_id,
                               const int64_t* tails_in, int64_t* tails_out, float* running_out,
                               int64_t* parents_out, int64_t* tokens_out, const uint32_t* seen_in, uint32_t* seen_out,
                               int64_t seen_stride_words, const int32_t* hist_in, int32_t* hist_out,
                               int64_t hist_stride, const uint32_t* whash_in, uint32_t* whash_out,
                               unsigned long long* guard_table, int64_t guard_entries, int32_t window, void* stream) {
  if (!picks || !pick_scores || !n_picks || !status || !running_out || !parents_out || !tokens_out) return SV_E_ARG;
  if (n_stop > 0 && (!stop_ids || !tails_in || !tails_out)) return SV_E_ARG;
  if ((seen_in == nullptr) != (seen_out == nullptr) || (hist_in == nullptr) != (hist_out == nullptr)) return SV_E_ARG;
  if (beams < 1 || vocab < 1 || num_picks < 1 || num_picks > kMaxPicks || beams > num_picks || step < 0 ||
      n_stop < 0 || n_stop > kMaxStop)
    return SV_E_SHAPE;
  const int64_t words = ((int64_t)vocab + 31) / 32;
  if (seen_in && seen_stride_words < words) return SV_E_SHAPE;
  if (tails_in && tails_in == tails_out) return SV_E_ARG;
  if (hist_in && (hist_stride <= step || hist_in == hist_out)) return SV_E_ARG;
  if (guard_table) {
    if (!hist_in || !whash_in || !whash_out || whash_in == whash_out) return SV_E_ARG;
    if (guard_entries < 2 || (guard_entries & (guard_entries - 1)) || window < 1 || window > 1024) return SV_E_SHAPE;
    if (reinterpret_cast<uintptr_t>(guard_table) % 8) return SV_E_ALIGN;
  }
  if (seen_in) {
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(seen_in), d0 = reinterpret_cast<uintptr_t>(seen_out);
    const uintptr_t span = (uintptr_t)beams * seen_stride_words * 4;
    if (s0 < d0 + span && d0 < s0 + span) return SV_E_ARG;
  }
  AdvanceArgs a;
  a.picks = picks;
  a.pick_scores = pick_scores;
  a.n_picks = n_picks;
  a.status = status;
  a.beams = beams;
  a.num_picks = num_picks;
  a.n_stop = n_stop;
  a.vocab = vocab;
  a.step = step;
  a.last = last != 0;
  a.stop_ids = stop_ids;
  a.eos_id = eos_id;
  a.tails_in = tails_in;
  a.tails_out = tails_out;
  a.running_out = running_out;
  a.parents_out = parents_out;
  a.tokens_out = tokens_out;
  a.seen_in = seen_in;
  a.seen_out = seen_out;
  a.seen_words = words;
  a.seen_stride = seen_stride_words;
  a.hist_in = hist_in;
  a.hist_out = hist_out;
  a.hist_stride = hist_stride;
  a.whash_in = whash_in;
  a.whash_out = whash_out;
  a.guard_table = guard_table;
  a.guard_mask = guard_entries - 1;
  a.window = window;
  // One block per ANT copied words, so each thread moves one word in one round trip
  // (every block repeats the small decision, which is cheaper than a second pass).
  const int64_t items = (seen_in ? (int64_t)beams * words : 0) + (hist_in ? (int64_t)beams * (step + 1) : 0);
  int64_t blocks = (items + ANT - 1) / ANT;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  beam_advance_kernel<<<(unsigned)blocks, ANT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? SV_OK : SV_E_CUDA;
}
