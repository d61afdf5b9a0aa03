/*
 * starvector_sampling.h -- C ABI of the B200 (sm_100a) decode-sampling kernels.
 *
 * A drop-in for the per-token sampling step of ComfyUI-StarVector-GGUF's native
 * generation loop (runtime_shared.py, `generate_tokens` :268 -> `_sample` :194 /
 * `_beam_sample` :214).  Every entry point:
 *   - takes plain device pointers and sizes (no framework types) and a CUDA
 *     stream (`stream`, a cudaStream_t; NULL = the legacy default stream);
 *   - enqueues its kernels on that stream and returns without synchronising,
 *     allocating or printing, so a call can be captured in a CUDA graph;
 *   - returns SV_OK or a negative SV_E_* code when an argument is invalid (then
 *     nothing is launched);
 *   - reports data-dependent failures per row through `out_status` (SV_ST_*).
 * Sizes: rows/beams >= 1, 1 <= vocab <= 524288, 1 <= top_k <= 128, 1 <= keep <= 128,
 * max(top_k, keep) <= vocab.
 */
#ifndef STARVECTOR_SAMPLING_H
#define STARVECTOR_SAMPLING_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes (argument errors; nothing launched). */
#define SV_OK 0
#define SV_E_ARG (-1)       /* null pointer or inconsistent arguments */
#define SV_E_DTYPE (-2)     /* unknown dtype / history kind / dense mode */
#define SV_E_SHAPE (-3)     /* rows, vocab, strides or capacities out of range */
#define SV_E_RANGE (-4)     /* temperature <= 0, top_p outside (0, 1], top_k/keep range */
#define SV_E_ALIGN (-5)     /* pointer not aligned to its element size */
#define SV_E_WORKSPACE (-6) /* workspace missing or smaller than required */
#define SV_E_CUDA (-7)      /* the CUDA launch itself failed */
#define SV_E_NOALLOC_LIMIT (-8) /* sv_beam_step_noalloc: beams x vocab beyond its fixed scratch */

/* Per-row status written by the kernels (out_status). */
#define SV_ST_OK 0
#define SV_ST_NAN 1        /* a NaN logit (the reference's multinomial raises) */
#define SV_ST_POSINF 2     /* +inf after penalty/temperature (softmax gives NaN) */
#define SV_ST_ALLNEGINF 3  /* no finite logit in the row */
#define SV_ST_HISTORY 4    /* a history id outside [0, vocab) */
#define SV_ST_TIMEOUT 5    /* a bounded wait on an asynchronous copy ran out */
#define SV_ST_SHARD_OVERFLOW 6 /* sv_merge_shards: a slice's kept list exceeded its capacity */
#define SV_ST_GUARD_FULL 7     /* sv_loop_guard_incremental: a window did not fit in the table */

/* Logit dtypes. */
#define SV_F32 0
#define SV_F16 1
#define SV_BF16 2

/* History kinds: the generated tokens the repetition penalty applies to. */
#define SV_HIST_NONE 0   /* no penalty */
#define SV_HIST_IDS32 1  /* int32 ids [rows, history_cols], valid prefix history_len[r] */
#define SV_HIST_IDS64 2  /* int64 ids, same layout */
#define SV_HIST_MASK8 3  /* bool/uint8 mask [rows, vocab] (the reference's `seen`) */
#define SV_HIST_BITS32 4 /* packed bitmap uint32 [rows, ceil(vocab/32)], bit i of word i/32 */

/* Dense output of sv_sample_step. */
#define SV_DENSE_NONE 0
#define SV_DENSE_SCORES 1 /* the warped scores: what _warp returns (-inf where masked) */
#define SV_DENSE_PROBS 2  /* softmax of the warped scores (0 where masked) */

/* Flags. */
#define SV_FLAG_FORCE_GENERAL 1 /* take the general (tie-group) path for every row */
#define SV_FLAG_CLUSTER 2       /* sv_sample_step: use the cluster kernel (rows split across CTAs) */
#define SV_FLAG_STREAM 4        /* sv_sample_step: use the streaming kernel (one CTA per row) */
#define SV_FLAG_TEST_WAIT_TIMEOUT 8 /* test hook (sv_sample_step, streaming kernel, id histories staged by
                                       bulk copy): the history copy's barrier expects 16 bytes more than
                                       the copy brings, so its bounded wait runs out after ~2 ms and every
                                       such row reports SV_ST_TIMEOUT; the copy itself lands */

/*
 * One sample-mode step for `rows` independent sequences.
 * Replaces, per row, runtime_shared.py:200-202:
 *     scores = _warp(_penalize(logits.float(), seen), temperature, top_p, 1)
 *     token  = torch.multinomial(scores.softmax(-1), 1); seen[token] = True
 * with the draw taken from the supplied uniform: the kept tokens in ascending
 * index order, the first whose inclusive prefix of fixed-point weights exceeds
 * floor(u * total).
 *   logits          [rows, row_stride] of dtype; row_stride 0 broadcasts one row
 *                   (the prefill's expanded logits, runtime_1b.py:82)
 *   history...      see SV_HIST_*; history_len may be NULL (= history_cols);
 *                   lengths are clamped to [0, history_cols]
 *   uniforms        float [rows] in [0, 1)
 *   temperature, top_p, repetition_penalty: doubles, cast to float as torch casts
 *                   a Python scalar; top-p is active iff top_p < 1, with
 *                   threshold float(1 - top_p) (runtime_shared.py:182-184)
 *   top_k, keep     runtime_shared.py:180 uses k = max(top_k, keep)
 *   out_token       int64 [rows] (-1 on a row error)
 *   out_count       int32 [rows] kept tokens (may be NULL)
 *   out_idx/out_prob/out_score  [rows, out_capacity]: the first out_capacity kept
 *                   tokens in ascending index order, their probability and warped
 *                   score (each may be NULL)
 *   out_dense       float [rows, dense_row_stride] per SV_DENSE_* (NULL if NONE)
 *   out_status      int32 [rows] (may be NULL)
 *   seen_bits_update  optional packed bitmap [rows, seen_bits_row_stride words]:
 *                   the drawn token's bit is set (runtime_shared.py:202)
 * Two kernels implement the same arithmetic: a streaming kernel (one persistent
 * CTA per SM walks its rows; chosen for many rows) and a cluster kernel (each row
 * split across a thread-block cluster; chosen for few rows or vocabularies whose
 * seen mask does not fit one CTA).  SV_FLAG_CLUSTER / SV_FLAG_STREAM force one.
 */
int sv_sample_step(const void* logits, int32_t logits_dtype, int32_t rows, int32_t vocab, int64_t logits_row_stride,
                   const void* history, int32_t history_kind, int64_t history_row_stride,
                   const int32_t* history_len, int32_t history_cols, const float* uniforms, double temperature,
                   double top_p, int32_t top_k, int32_t keep, double repetition_penalty, int64_t* out_token,
                   int32_t* out_count, int32_t* out_idx, float* out_prob, float* out_score, int32_t out_capacity,
                   float* out_dense, int32_t dense_mode, int64_t dense_row_stride, int32_t* out_status,
                   uint32_t* seen_bits_update, int64_t seen_bits_row_stride, int32_t flags, void* stream);

/* Workspace bytes sv_beam_step needs for `beams` x `vocab`.  The workspace must be
 * zero-filled once before its first use; the kernel leaves it reusable. */
size_t sv_beam_workspace_bytes(int32_t beams, int32_t vocab);

/*
 * One beam-sampling step (runtime_shared.py:230-237):
 *     log_probs = _warp(_penalize(log_softmax(logits.float()), seen), T, top_p, 2)
 *     scores    = (log_probs + running_scores[:, None]).view(1, -1)
 *     picks     = multinomial(scores.softmax(-1), min(num_picks, count_nonzero))
 * Draws without replacement from `uniforms[0..num_picks)`: pick j is the first
 * remaining entry (flattened beam*vocab order) whose inclusive prefix weight
 * exceeds floor(u_j * remaining total).  The host keeps the divmod, finishing,
 * length penalty and ordering logic (runtime_shared.py:237-260).
 *   running_scores  float [beams]; uniforms float [num_picks]; num_picks <= 64
 *   out_picks       int64 [num_picks] flattened indices b*vocab + token
 *   out_pick_scores float [num_picks] = scores at the picks (:236)
 *   out_num_picks   int32 [1]; out_status int32 [1]
 *   out_kept_*      optional per-beam kept tokens [beams, out_capacity] (index
 *                   order): ids, warped log-probs, probabilities over beams*vocab
 *   out_dense_logprob optional float [beams, dense_row_stride]: log_probs as above
 */
int sv_beam_step(const void* logits, int32_t logits_dtype, int32_t beams, int32_t vocab, int64_t logits_row_stride,
                 const void* history, int32_t history_kind, int64_t history_row_stride, const int32_t* history_len,
                 int32_t history_cols, const float* running_scores, const float* uniforms, int32_t num_picks,
                 double temperature, double top_p, int32_t top_k, int32_t keep, double repetition_penalty,
                 int64_t* out_picks, float* out_pick_scores, int32_t* out_num_picks, int32_t* out_status,
                 int32_t* out_kept_count, int32_t* out_kept_idx, float* out_kept_logprob, float* out_kept_prob,
                 int32_t out_capacity, float* out_dense_logprob, int64_t dense_row_stride, void* workspace,
                 size_t workspace_bytes, int32_t flags, void* stream);

/*
 * sv_beam_step_noalloc: sv_beam_step for callers that cannot allocate device
 * memory.  No counterpart in the reference (its beam step allocates through torch).
 * A host application that owns the GPU's memory and forbids plugins to allocate, or
 * a loop that must not allocate during a step, cannot provide sv_beam_step's
 * workspace; this variant uses a fixed 8 MiB array that the library declares in
 * device memory instead (held by every GPU that loads the library until the
 * process exits).  Arguments and results are sv_beam_step's, without the workspace.
 * Limit: sv_beam_workspace_bytes(beams, vocab) <= 8 MiB, i.e. beams * vocab <=
 * 524271 (8 beams up to vocab 65533); larger calls return SV_E_NOALLOC_LIMIT.
 * The first call on a device looks up the array's device address (make it before
 * any stream capture) and keeps it for the life of the process: after
 * cudaDeviceReset, or anything else that replaces the device's primary context,
 * that address is stale, so the entry point must not be called again on that
 * device.  Each call clears the array's header on `stream`.  All calls share the
 * array: calls that overlap on the GPU race.
 */
int sv_beam_step_noalloc(const void* logits, int32_t logits_dtype, int32_t beams, int32_t vocab,
                         int64_t logits_row_stride, const void* history, int32_t history_kind,
                         int64_t history_row_stride, const int32_t* history_len, int32_t history_cols,
                         const float* running_scores, const float* uniforms, int32_t num_picks, double temperature,
                         double top_p, int32_t top_k, int32_t keep, double repetition_penalty, int64_t* out_picks,
                         float* out_pick_scores, int32_t* out_num_picks, int32_t* out_status,
                         int32_t* out_kept_count, int32_t* out_kept_idx, float* out_kept_logprob,
                         float* out_kept_prob, int32_t out_capacity, float* out_dense_logprob,
                         int64_t dense_row_stride, int32_t flags, void* stream);

/*
 * Loop guard for `rows` token histories (runtime_shared.py:156-167, `_repeating`):
 * verdict[r] = 1 iff lengths[r] >= window*repeats and the last `window` tokens of
 * row r occur at least `repeats` times.  tokens int32 or int64 (token_bytes 4/8)
 * [rows, row_stride]; 1 <= window <= 1024.  lengths[r] is clamped to row_stride
 * when row_stride > 0, and then every row must hold row_stride readable elements
 * (the kernel may read a row's whole stride before it knows the row's length);
 * with row_stride 0 the caller guarantees the length.
 */
int sv_loop_guard(const void* tokens, int32_t token_bytes, int32_t rows, int64_t row_stride, const int32_t* lengths,
                  int32_t window, int32_t repeats, uint8_t* out_verdict, void* stream);

/* The reference's _penalize on its own (runtime_shared.py:170-173): out =
 * seen ? (x < 0 ? x*p : x/p) : x as float [rows, out_row_stride]; history kinds
 * SV_HIST_MASK8 or SV_HIST_BITS32. */
int sv_penalize(const void* logits, int32_t logits_dtype, int32_t rows, int32_t vocab, int64_t logits_row_stride,
                const void* history, int32_t history_kind, int64_t history_row_stride, double repetition_penalty,
                float* out, int64_t out_row_stride, void* stream);

/* seen[r, tokens[r]] = 1 on a packed bitmap (runtime_shared.py:202). */
int sv_seen_update(uint32_t* seen_bits, int32_t rows, int64_t row_stride_words, const int64_t* tokens,
                   int32_t vocab, void* stream);

/* dst[b] = src[parents[b]] with bit tokens[b] set (runtime_shared.py:258-259);
 * tokens may be NULL.  src and dst must not overlap. */
int sv_seen_reorder(const uint32_t* src, uint32_t* dst, int32_t beams, int32_t vocab, int64_t row_stride_words,
                    const int64_t* parents, const int64_t* tokens, void* stream);

/*
 * Vocab-sharded sample step, merge side.  No single counterpart in the reference:
 * it replaces runtime_shared.py:180-186 and :201 (top-k with ties, top-p, the draw)
 * for a row whose vocabulary is split across ranks, each rank having run
 * sv_sample_step on its slice with top_p = 1 and out_capacity = capacity (its kept
 * list is then the slice's top-k with ties).  `packed` holds, for each of `shards`
 * slices and each row, one int32 record of 2 * capacity + 2 values:
 *   [0, capacity)             the kept tokens' warped scores (float bits, out_score)
 *   [capacity, 2 * capacity)  their global indices (out_idx + the slice's offset)
 *   2 * capacity              the slice's kept count (out_count)
 *   2 * capacity + 1          the slice's status (out_status)
 * laid out [shards][rows][record] (what an all-gather of each rank's [rows][record]
 * produces).  Results equal sv_sample_step on the whole row with the same
 * uniforms.  shards * capacity <= 1024; max(top_k, keep) <= capacity.  A row whose
 * slice kept more than `capacity` tokens (a tie group) gets SV_ST_SHARD_OVERFLOW and
 * must be sampled unsharded.
 *   out_token int64 [rows]; out_count int32 [rows] (may be NULL); out_idx / out_prob
 *   [rows, out_capacity] the kept tokens in index order and their probabilities
 *   (may be NULL); out_status int32 [rows] (may be NULL)
 */
int sv_merge_shards(const int32_t* packed, int32_t shards, int32_t rows, int32_t capacity, const float* uniforms,
                    double top_p, int32_t top_k, int32_t keep, int64_t* out_token, int32_t* out_count,
                    int32_t* out_idx, float* out_prob, int32_t out_capacity, int32_t* out_status, void* stream);

/* Vocab-sharded sample step, one rank's side of the exchange: its records
 * [rows][2 * capacity + 2] (the layout sv_merge_shards reads) from its slice step's
 * out_count, out_status, out_idx and out_score ([rows, capacity]), with the slice's
 * offset added to the ids.  No counterpart in the reference (it has no sharded
 * vocabulary). */
int sv_pack_slice(const int32_t* count, const int32_t* status, const int32_t* idx, const float* score, int32_t rows,
                  int32_t capacity, int32_t offset, int32_t* out_records, void* stream);

/*
 * Vocab-sharded beam step.  No counterpart in the reference (it has no sharded
 * vocabulary); together these replace runtime_shared.py:230-235 for beams whose
 * vocabulary is split across ranks.  Each rank owns the same slice of every
 * beam's row:
 *   1. sv_beam_slice_stats with global_max = NULL: out_max [beams] the slice's
 *      maximum (NaN-propagating), out_flags [beams] 2 for a NaN in the slice, else
 *      1 for a +inf, else 0.  The ranks all-reduce both with MAX.
 *   2. sv_beam_slice_stats with global_max = the reduced maxima: out_sum [beams]
 *      the slice's exact sum of trunc(exp(x - M) * 2^44).  The ranks all-reduce it
 *      with SUM (int64: the sum wraps the same on every rank).
 *   3. sv_beam_slice_logprobs: the slice's log_softmax (x - M) - ln(sum * 2^-44),
 *      float32 [beams, out_row_stride], as sv_beam_step forms it.
 *   4. sv_sample_step on those log-probs with top_p = 1, keep = 2 and out_capacity
 *      = capacity (penalty, temperature and the slice's top-k with ties), then
 *      sv_pack_slice; the ranks all-gather the records.
 *   5. sv_merge_beam_shards: per beam the exact top-k with ties and top-p over the
 *      union, then + running scores, the softmax over all beams' kept entries,
 *      count_nonzero and the draws without replacement, as sv_beam_step.  Results
 *      equal sv_beam_step on the whole rows.  global_max / global_flags are the
 *      reduced statistics of step 1 (they carry the log_softmax stage's status);
 *      vocab is the whole row's size (picks are beam * vocab + token); workspace
 *      holds sv_merge_beam_shards_workspace_bytes(beams, shards, capacity) bytes,
 *      16-byte aligned (no zero-fill needed).  Outputs as sv_beam_step.
 * logits [beams, slice_len] at logits_row_stride elements; beams <= 32.
 */
int sv_beam_slice_stats(const void* logits, int32_t logits_dtype, int32_t beams, int32_t slice_len,
                        int64_t logits_row_stride, const float* global_max, float* out_max, int32_t* out_flags,
                        uint64_t* out_sum, void* stream);
int sv_beam_slice_logprobs(const void* logits, int32_t logits_dtype, int32_t beams, int32_t slice_len,
                           int64_t logits_row_stride, const float* global_max, const uint64_t* global_sum, float* out,
                           int64_t out_row_stride, void* stream);
size_t sv_merge_beam_shards_workspace_bytes(int32_t beams, int32_t shards, int32_t capacity);
int sv_merge_beam_shards(const int32_t* packed, int32_t shards, int32_t beams, int32_t capacity, int32_t vocab,
                         const float* global_max, const int32_t* global_flags, const float* running_scores,
                         const float* uniforms, int32_t num_picks, double top_p, int32_t top_k, int32_t keep,
                         void* workspace, size_t workspace_bytes, int64_t* out_picks, float* out_pick_scores,
                         int32_t* out_num_picks, int32_t* out_status, int32_t* out_kept_count, int32_t* out_kept_idx,
                         float* out_kept_logprob, float* out_kept_prob, int32_t out_capacity, void* stream);

/*
 * The same merges over slice blocks, the exchange layout a rank's sv_sample_step
 * (or its beam slice step) writes directly, so no packing launch is needed.  No
 * counterpart in the reference (it has no sharded vocabulary).  Each shard's block
 * is int32 [2 * rows * capacity + 2 * rows]:
 *   [0, rows * capacity)                    out_score [rows][capacity] (float bits)
 *   [rows * capacity, 2 * rows * capacity)  out_idx [rows][capacity], slice-local
 *   [2 * rows * capacity, + rows)           out_count [rows]
 *   [2 * rows * capacity + rows, + rows)    out_status [rows]
 * and `blocks` holds the shards' blocks back to back (an all-gather of each rank's
 * block).  Shard s's indices are offset by s * slice_stride (its slice starts
 * there).  Otherwise as sv_merge_shards / sv_merge_beam_shards.
 */
int sv_merge_slices(const int32_t* blocks, int32_t shards, int32_t rows, int32_t capacity, int32_t slice_stride,
                    const float* uniforms, double top_p, int32_t top_k, int32_t keep, int64_t* out_token,
                    int32_t* out_count, int32_t* out_idx, float* out_prob, int32_t out_capacity, int32_t* out_status,
                    void* stream);
int sv_merge_beam_slices(const int32_t* blocks, int32_t shards, int32_t beams, int32_t capacity, int32_t slice_stride,
                         int32_t vocab, const float* global_max, const int32_t* global_flags,
                         const float* running_scores, const float* uniforms, int32_t num_picks, double top_p,
                         int32_t top_k, int32_t keep, void* workspace, size_t workspace_bytes, int64_t* out_picks,
                         float* out_pick_scores, int32_t* out_num_picks, int32_t* out_status,
                         int32_t* out_kept_count, int32_t* out_kept_idx, float* out_kept_logprob,
                         float* out_kept_prob, int32_t out_capacity, void* stream);

/*
 * Beam KV-cache reorder (replaces runtime_shared.py:388-394, CachedDecoding.reorder):
 * every beam row r whose parent parents[r] differs from r receives its parent's
 * keys and values over the first `length` cache slots, as the reference's
 * keys[:, rows, ..., :length, :] = keys[:, sources, ..., :length, :] (sources read
 * before rows are written, so swaps are safe); rows whose parent is themselves are
 * not touched.  parents int64 [beams] in device memory (no host sync: the beam
 * step's picks can feed it directly).  keys and values (values may be NULL) share
 * one layout: element (layer, beam, head, slot, d) at
 *   layer * stride_layer + beam * stride_beam + head * stride_head + slot * stride_slot + d
 * (strides in elements; the 1B decoder's MQA cache [layers, beams, capacity, head_dim]
 * has heads = 1, the 8B decoder's GQA cache [layers, beams, kv_heads, capacity,
 * head_dim] heads = kv_heads).  elem_bytes 1, 2 or 4; head_dim * elem_bytes, every
 * stride in bytes and both pointers must be multiples of 16; beams <= 8 (the
 * node's num_beams maximum, nodes.py:128); layers * heads <= 65535;
 * length * head_dim * elem_bytes < 2^34.  out_status (may be NULL) int32: 1 when a parent lies
 * outside [0, beams) (its row is left as it is), else 0.  No counterpart of the
 * kernel in the reference (it indexes with torch).
 */
int sv_kv_reorder(void* keys, void* values, int32_t elem_bytes, int32_t layers, int32_t beams, int32_t heads,
                  int64_t length, int32_t head_dim, int64_t stride_layer, int64_t stride_beam, int64_t stride_head,
                  int64_t stride_slot, const int64_t* parents, int32_t* out_status, void* stream);

/*
 * Incremental loop guard (runtime_shared.py:156-167, `_repeating`, checked every 16
 * steps at :207 and :254) for one growing sequence: the verdict of sv_loop_guard in
 * time independent of the sequence's length.  `table` (table_entries, a power of
 * two, 8-byte words; all bits set = empty, fill it with 0xFF before the first call)
 * holds one entry per (window hash, start) of the sequence's windows.  The call
 * first inserts the windows ending at positions [insert_from, length) of `tokens`
 * (int32 or int64, the sequence's first `length` tokens), then counts the starts
 * whose `window` tokens equal the last `window` (hash matches verified token by
 * token): out_verdict = length >= window * repeats && count >= repeats.  Calling it
 * with insert_from = the previous call's length keeps every window in the table.
 * The beam loop inserts its rows' windows inside sv_beam_advance instead (then
 * insert_from = length).  Size the table to at least twice the windows inserted;
 * out_status (may be NULL) gets SV_ST_GUARD_FULL if an insert found no slot.
 * 1 <= window <= 1024; one CTA.
 */
int sv_loop_guard_incremental(unsigned long long* table, int64_t table_entries, const void* tokens,
                              int32_t token_bytes, int64_t insert_from, int64_t length, int32_t window,
                              int32_t repeats, uint8_t* out_verdict, int32_t* out_status, void* stream);

/*
 * The beam loop's per-step decision on the device (replaces the host bookkeeping
 * of runtime_shared.py:237-259 that decides the next step; the finished list, stop
 * tests and loop guard stay with the caller).  Inputs are one sv_beam_step's
 * outputs (picks beam * vocab + token, pick_scores, n_picks, status; num_picks
 * slots).  With hits[j] = last || token_j == eos_id || the candidate (parent row's
 * tokens + token_j, step + 1 long) ends with stop_ids[0..n_stop), live[j] =
 * (double)pick_scores[j] - 1e9 * hits[j] and order = the first `beams` picks by
 * live descending (ties in pick order), padded with order[0]:
 *   running_out[r] = (float)live[order[r]] (or -1e9 past the n picks),
 *   parents_out[r] = parent of order[r], tokens_out[r] = token of order[r],
 *   tails_out[r]   = tails_in[parent] shifted by one, token appended
 *                    (tails int64 [beams, n_stop], each running row's last n_stop
 *                    tokens, -1 before the sequence starts; unused when n_stop = 0),
 *   seen_out[r]    = seen_in[parent] with the token's bit set (optional: both NULL
 *                    to skip; packed bitmaps, row stride seen_stride_words),
 *   hist_out[r]    = hist_in[parent][0, step) then the token (optional: both NULL
 *                    to skip; int32 rows of hist_stride > step entries, the running
 *                    rows' generated tokens, for the loop guard),
 *   whash_out[r]   = the row's rolling hash of its last `window` tokens (uint32
 *                    [beams], zero before the first step), its window entered in
 *                    guard_table once step >= window - 1 (optional: guard_table
 *                    NULL to skip; needs the histories; the table layout and sizing
 *                    are sv_loop_guard_incremental's, whose probe with
 *                    insert_from = length then checks running row 0).
 * A step whose status is non-zero, or without a valid pick, leaves every row its
 * own state (parents r, tokens 0, running 0 / -1e9).  eos_id -1 never matches.
 * beams <= num_picks <= 64, n_stop <= 16; tails_in != tails_out, hist_in != hist_out;
 * seen_in and seen_out must not overlap.  All pointers device memory; nothing is read on the host.
 */
int sv_beam_advance(const int64_t* picks, const float* pick_scores, const int32_t* n_picks, const int32_t* status,
                    int32_t beams, int32_t vocab, int32_t num_picks, int32_t step, int32_t last,
                    const int64_t* stop_ids, int32_t n_stop, int64_t eos_id, const int64_t* tails_in,
                    int64_t* tails_out, float* running_out, int64_t* parents_out, int64_t* tokens_out,
                    const uint32_t* seen_in, uint32_t* seen_out, int64_t seen_stride_words, const int32_t* hist_in,
                    int32_t* hist_out, int64_t hist_stride, const uint32_t* whash_in, uint32_t* whash_out,
                    unsigned long long* guard_table, int64_t guard_entries, int32_t window, void* stream);

/* Text of a return or status code. */
const char* sv_error_string(int32_t code);

/* ABI version of this library. */
int32_t sv_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* STARVECTOR_SAMPLING_H */
