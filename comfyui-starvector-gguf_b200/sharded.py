"""Multi-GPU sampling over torch.distributed, one process per GPU.

Row-sharded.  Rows are independent sequences (runtime_shared.py:268-342 runs one
sequence, or one beam group, per call): each rank samples its own contiguous block
of rows (`row_block`) with ops.sample_step.  There is no collective in the step.

Vocab-sharded.  A row's vocabulary is split across ranks (as behind a
vocab-parallel lm_head), each rank holding the slice [offset, offset + width), the
slices `slice_stride` apart.  Each rank keeps its slice's top-k with ties
(runtime_shared.py:172-181 on the slice: sv_sample_step with top_p = 1 and a
kept-list capacity), writing it straight into its exchange block (scores,
slice-local ids, counts, statuses: the sv_merge_slices layout).  One all-gather
exchanges the blocks (NCCL over NVLink), and every rank merges them into the same
token (sv_merge_slices: the k-th largest with ties, top-p, the draw,
runtime_shared.py:180-186 and :201).  The result equals the unsharded step on the
whole row.  The penalty's history comes as the row's seen bitmap (or bool mask), of
which each rank reads its slice; slice offsets are multiples of 32.

`VocabShardedSampler` and `VocabShardedBeamStep` keep every buffer of a step and
capture it (slice kernels, collectives, merge) as one CUDA graph per rank, for a
decode loop that replays the same step each token.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def row_block(rows: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous rows [lo, hi) that `rank` of `world` samples."""
    per = (rows + world - 1) // world
    lo = min(rank * per, rows)
    return lo, min(lo + per, rows)


def slice_bounds(vocab: int, rank: int, world: int) -> tuple[int, int, int]:
    """(offset, width, slice_stride) of `rank`'s vocabulary slice: slices of a
    multiple of 32 tokens (the seen bitmap's word), the last one shorter."""
    stride = ((vocab + world - 1) // world + 31) // 32 * 32
    offset = min(rank * stride, vocab)
    return offset, min(stride, vocab - offset), stride


def slice_step(shard_logits, uniforms, *, offset, seen_bits=None, seen=None, temperature=1.5, top_k=50, keep=1,
               repetition_penalty=3.1, capacity=64, out=None):
    """One rank's part before the exchange: its slice's top-k with ties.

    shard_logits [rows, width] (the vocabulary slice at `offset`); seen_bits the
    whole row's packed bitmap [rows, ceil(vocab / 32)] or seen the whole row's bool
    mask [rows, vocab] (each optional).  Returns sample_step's outputs (kept ids in
    slice coordinates, warped scores, count, status), in `out` when given (an
    exchange block's views, ops.slice_block_outputs).
    """
    width = shard_logits.shape[-1]
    kw = {}
    if seen_bits is not None:
        if offset % 32:
            raise ValueError("slice offsets must be multiples of 32 (the seen bitmap's word size)")
        kw["seen_bits"] = seen_bits[:, offset // 32: offset // 32 + (width + 31) // 32]
    elif seen is not None:
        kw["seen"] = seen[:, offset: offset + width]
    return ops.sample_step(shard_logits, uniforms, temperature=temperature, top_p=1.0, top_k=top_k, keep=keep,
                           repetition_penalty=repetition_penalty, out_capacity=capacity, out=out, **kw)


def fill_block(block, local, rows, capacity):
    """A slice step's outputs (count, status, idx, score [rows, capacity]) written
    into an exchange block (for slice steps that did not write it directly)."""
    RC = rows * capacity
    block[:RC] = local["score"].reshape(-1).view(torch.int32)
    block[RC:2 * RC] = local["idx"].reshape(-1)
    block[2 * RC:2 * RC + rows] = local["count"]
    block[2 * RC + rows:] = local["status"]
    return block


def all_gather_blocks(block, group=None):
    """[world, block_len] exchange blocks of every rank (rank order)."""
    world = dist.get_world_size(group)
    out = torch.empty((world, block.numel()), dtype=block.dtype, device=block.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(-1), block, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), block, group=group)
    return out


def _slice_into_block(step_fn, shard_logits, uniforms, rows, capacity, offset, **kw):
    block = torch.empty(ops.block_len(rows, capacity), dtype=torch.int32, device=shard_logits.device)
    if step_fn is None and block.is_cuda:
        slice_step(shard_logits, uniforms, offset=offset, capacity=capacity,
                   out=ops.slice_block_outputs(block, rows, capacity), **kw)
    else:
        local = (step_fn or slice_step)(shard_logits, uniforms, offset=offset, capacity=capacity, **kw)
        fill_block(block, local, rows, capacity)
    return block


def sample_step_vocab_sharded(shard_logits, uniforms, *, offset, slice_stride=None, seen_bits=None, seen=None,
                              temperature=1.5, top_p=0.9, top_k=50, keep=1, repetition_penalty=3.1, capacity=64,
                              out_capacity=0, group=None, step_fn=None, merge_fn=None, out=None):
    """The vocab-sharded sample step, called by every rank of `group` with its slice
    (slices `slice_stride` apart; default: this slice's width, for equal slices).

    Every rank returns the same dict: token int64 [rows], count int32 [rows], status
    int32 [rows] (SV_ST_SHARD_OVERFLOW where a slice's tie group outgrew
    `capacity`: sample that row unsharded), and idx / prob [rows, out_capacity].
    step_fn / merge_fn replace slice_step / ops.merge_shards (the tests use them to
    run the exchange on CPU ranks).
    """
    R = shard_logits.shape[0]
    stride = shard_logits.shape[-1] if slice_stride is None else int(slice_stride)
    block = _slice_into_block(step_fn, shard_logits, uniforms, R, capacity, offset, seen_bits=seen_bits, seen=seen,
                              temperature=temperature, top_k=top_k, keep=keep,
                              repetition_penalty=repetition_penalty)
    blocks = all_gather_blocks(block, group)
    return (merge_fn or ops.merge_shards)(blocks, uniforms, capacity=capacity, top_p=top_p, top_k=top_k, keep=keep,
                                          out_capacity=out_capacity, out=out, rows=R, slice_stride=stride)


def beam_step_vocab_sharded(shard_logits, running_scores, uniforms, *, offset, vocab, slice_stride=None,
                            seen_bits=None, seen=None, temperature=1.5, top_p=0.9, top_k=50, keep=2,
                            repetition_penalty=3.1, capacity=64, num_picks=None, out_capacity=0, group=None,
                            stats_fn=None, logprob_fn=None, step_fn=None, merge_fn=None, out=None):
    """The vocab-sharded beam step (runtime_shared.py:230-235), called by every rank
    of `group` with its slice [beams, width] of every beam's logits at `offset`.

    Three exchanges: the slices' maxima and NaN / +inf flags (all-reduce MAX), their
    exact fixed-point exp sums against the global maximum (all-reduce SUM, int64),
    then the slices' kept lists (all-gather of the exchange blocks).  Between them
    each rank forms its slice's log_softmax and runs the slice step on it (penalty,
    temperature, the slice's top-k with ties; top-p off).  Every rank returns
    beam_step's dict for the whole rows (picks are beam * vocab + token).  stats_fn /
    logprob_fn / step_fn / merge_fn replace the CUDA calls (the tests run the
    exchange on CPU ranks with them).
    """
    B = shard_logits.shape[0]
    stride = shard_logits.shape[-1] if slice_stride is None else int(slice_stride)
    stats = stats_fn or ops.beam_slice_stats
    first = stats(shard_logits)  # fresh tensors: reduced in place
    gmax, gflags = first["max"], first["flags"]
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(gflags, op=dist.ReduceOp.MAX, group=group)
    gsum = stats(shard_logits, global_max=gmax)["sum"]
    dist.all_reduce(gsum, op=dist.ReduceOp.SUM, group=group)
    lp = (logprob_fn or ops.beam_slice_logprobs)(shard_logits, gmax, gsum)
    dummy = torch.zeros(B, dtype=torch.float32, device=lp.device)
    block = _slice_into_block(step_fn, lp, dummy, B, capacity, offset, seen_bits=seen_bits, seen=seen,
                              temperature=temperature, top_k=top_k, keep=keep,
                              repetition_penalty=repetition_penalty)
    blocks = all_gather_blocks(block, group)
    return (merge_fn or ops.merge_beam_shards)(blocks, gmax, gflags, running_scores, uniforms, capacity=capacity,
                                               vocab=vocab, top_p=top_p, top_k=top_k, keep=keep,
                                               num_picks=num_picks, out_capacity=out_capacity, out=out, beams=B,
                                               slice_stride=stride)


class _GraphStep:
    """Runs `_run` eagerly or, after capture(), as one CUDA graph replay."""

    graph = None

    def capture(self, warmup=2):
        """Runs the step `warmup` times (the collectives set up their
        communicators) and captures it; later calls replay the graph."""
        stream = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._run()
        stream.wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self._run()
        self.graph = g
        return self

    def release(self):
        """Drops the graph (before the process group is destroyed)."""
        self.graph = None

    def __call__(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self._run()
        return self.out


class VocabShardedSampler(_GraphStep):
    """The vocab-sharded sample step bound to fixed input tensors (the decode
    loop's logits slice, uniforms and seen bitmap, updated in place between
    steps), with its exchange block, gathered blocks and outputs kept, so that the
    whole step can be captured as one CUDA graph (capture()).  Calling it runs the
    step and returns the output dict (the same tensors every call)."""

    def __init__(self, shard_logits, uniforms, *, offset, slice_stride=None, seen_bits=None, seen=None,
                 temperature=1.5, top_p=0.9, top_k=50, keep=1, repetition_penalty=3.1, capacity=64, out_capacity=0,
                 group=None):
        self.x, self.u = shard_logits, uniforms
        self.device = shard_logits.device
        R = shard_logits.shape[0]
        self.rows, self.capacity, self.offset = R, capacity, offset
        self.stride = shard_logits.shape[-1] if slice_stride is None else int(slice_stride)
        self.hist = dict(seen_bits=seen_bits, seen=seen)
        self.settings = dict(temperature=temperature, top_k=top_k, keep=keep, repetition_penalty=repetition_penalty)
        self.top_p, self.top_k, self.keep, self.out_capacity, self.group = top_p, top_k, keep, out_capacity, group
        world = dist.get_world_size(group)
        self.block = torch.empty(ops.block_len(R, capacity), dtype=torch.int32, device=self.device)
        self.local = ops.slice_block_outputs(self.block, R, capacity)
        self.blocks = torch.empty((world, self.block.numel()), dtype=torch.int32, device=self.device)
        self.out = {}

    def _run(self):
        slice_step(self.x, self.u, offset=self.offset, capacity=self.capacity, out=self.local, **self.hist,
                   **self.settings)
        dist.all_gather_into_tensor(self.blocks.view(-1), self.block, group=self.group)
        ops.merge_shards(self.blocks, self.u, capacity=self.capacity, top_p=self.top_p, top_k=self.top_k,
                         keep=self.keep, out_capacity=self.out_capacity, out=self.out, rows=self.rows,
                         slice_stride=self.stride)


# Beam groups whose whole logits are at most this many bytes are gathered whole
# (one all-gather, then the unsharded beam kernel on every rank) rather than
# exchanged as slice statistics and kept lists (three collectives).
GATHER_BEAM_BYTES = 8 << 20


class VocabShardedBeamStep(_GraphStep):
    """The vocab-sharded beam step bound to fixed input tensors (every beam's logits
    slice, running scores, uniforms and seen bitmap, updated in place between
    steps), with every intermediate kept, so that the whole step can be captured
    as one CUDA graph (capture()).

    method "gather": one all-gather of the slices, then sv_beam_step on the whole
    rows on every rank (for small beam groups: one collective).  method "exchange":
    the slice statistics and their two all-reduces, the slice log-probs and slice
    step, the all-gather of the kept lists and the merge (for rows too large to
    gather).  "auto" gathers when the whole logits take at most GATHER_BEAM_BYTES.
    Both give sv_beam_step's results on the whole rows."""

    def __init__(self, shard_logits, running_scores, uniforms, *, offset, vocab, slice_stride=None, seen_bits=None,
                 seen=None, temperature=1.5, top_p=0.9, top_k=50, keep=2, repetition_penalty=3.1, capacity=64,
                 num_picks=None, out_capacity=0, group=None, method="auto"):
        self.x, self.running, self.u = shard_logits, running_scores, uniforms
        self.device = shard_logits.device
        B, W = shard_logits.shape
        self.beams, self.capacity, self.offset, self.vocab = B, capacity, offset, vocab
        self.stride = W if slice_stride is None else int(slice_stride)
        self.hist = dict(seen_bits=seen_bits, seen=seen)
        self.settings = dict(temperature=temperature, top_k=top_k, keep=keep, repetition_penalty=repetition_penalty)
        self.top_p, self.top_k, self.keep, self.group = top_p, top_k, keep, group
        self.num_picks, self.out_capacity = num_picks, out_capacity
        world = dist.get_world_size(group)
        dev = self.device
        if method == "auto":
            method = "gather" if B * world * self.stride * shard_logits.element_size() <= GATHER_BEAM_BYTES \
                else "exchange"
        self.method = method
        self.out = {}
        if method == "gather":
            # Each rank's slice padded to the stride (-inf past the vocabulary), the
            # gathered slices, and the whole rows they are copied back into.
            self.send = torch.full((B, self.stride), float("-inf"), dtype=shard_logits.dtype, device=dev)
            self.gathered = torch.empty((world, B, self.stride), dtype=shard_logits.dtype, device=dev)
            self.whole = torch.empty((B, world * self.stride), dtype=shard_logits.dtype, device=dev)
            self.ws = ops.beam_workspace(B, vocab, dev)
            return
        if method != "exchange":
            raise ValueError("method must be 'auto', 'gather' or 'exchange'")
        self.stats = {"max": torch.empty(B, dtype=torch.float32, device=dev),
                      "flags": torch.empty(B, dtype=torch.int32, device=dev),
                      "sum": torch.empty(B, dtype=torch.int64, device=dev)}
        self.lp = torch.empty((B, W), dtype=torch.float32, device=dev)
        self.dummy = torch.zeros(B, dtype=torch.float32, device=dev)
        self.block = torch.empty(ops.block_len(B, capacity), dtype=torch.int32, device=dev)
        self.local = ops.slice_block_outputs(self.block, B, capacity)
        self.blocks = torch.empty((world, self.block.numel()), dtype=torch.int32, device=dev)
        nbytes = ops.L.lib().sv_merge_beam_shards_workspace_bytes(B, world, capacity)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def _run(self):
        if self.method == "gather":
            W = self.x.shape[1]
            self.send[:, :W].copy_(self.x)
            dist.all_gather_into_tensor(self.gathered.view(-1), self.send.view(-1), group=self.group)
            self.whole.view(self.beams, -1, self.stride).copy_(self.gathered.permute(1, 0, 2))
            ops.beam_step(self.whole[:, :self.vocab], self.running, self.u, top_p=self.top_p, num_picks=self.num_picks,
                          out_capacity=self.out_capacity, workspace=self.ws, out=self.out, **self.hist,
                          **self.settings)
            return
        st, g = self.stats, self.group
        ops.beam_slice_stats(self.x, out=st)
        dist.all_reduce(st["max"], op=dist.ReduceOp.MAX, group=g)
        dist.all_reduce(st["flags"], op=dist.ReduceOp.MAX, group=g)
        ops.beam_slice_stats(self.x, global_max=st["max"], out=st)
        dist.all_reduce(st["sum"], op=dist.ReduceOp.SUM, group=g)
        ops.beam_slice_logprobs(self.x, st["max"], st["sum"], out=self.lp)
        slice_step(self.lp, self.dummy, offset=self.offset, capacity=self.capacity, out=self.local, **self.hist,
                   **self.settings)
        dist.all_gather_into_tensor(self.blocks.view(-1), self.block, group=g)
        ops.merge_beam_shards(self.blocks, st["max"], st["flags"], self.running, self.u, capacity=self.capacity,
                              vocab=self.vocab, top_p=self.top_p, top_k=self.top_k, keep=self.keep,
                              num_picks=self.num_picks, out_capacity=self.out_capacity, workspace=self.ws,
                              out=self.out, beams=self.beams, slice_stride=self.stride)
