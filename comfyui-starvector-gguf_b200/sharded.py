"""Multi-GPU sampling over torch.distributed, one process per GPU.

Row-sharded.  Rows are independent sequences (runtime_shared.py:268-342 runs one
sequence, or one beam group, per call): each rank samples its own contiguous block
of rows (`row_block`) with ops.sample_step.  There is no collective in the step.

Vocab-sharded.  A row's vocabulary is split across ranks (as behind a
vocab-parallel lm_head), each rank holding the slice [offset, offset + width).
Each rank keeps its slice's top-k with ties (runtime_shared.py:172-181 on the
slice: sv_sample_step with top_p = 1 and a kept-list capacity).  One all-gather
exchanges those lists (NCCL over NVLink), and every rank merges them into the same
token (sv_merge_shards: the k-th largest with ties, top-p, the draw,
runtime_shared.py:180-186 and :201).  The result equals the unsharded step on the
whole row.  The penalty's history comes as the row's seen bitmap (or bool mask),
of which each rank reads its slice; slice offsets are multiples of 32.
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


def record_width(capacity: int) -> int:
    """int32 values per row in the exchanged records."""
    return 2 * capacity + 2


def slice_step(shard_logits, uniforms, *, offset, seen_bits=None, seen=None, temperature=1.5, top_k=50, keep=1,
               repetition_penalty=3.1, capacity=64):
    """One rank's part before the exchange: its slice's top-k with ties.

    shard_logits [rows, width] (the vocabulary slice at `offset`); seen_bits the
    whole row's packed bitmap [rows, ceil(vocab / 32)] or seen the whole row's bool
    mask [rows, vocab] (each optional).  Returns sample_step's outputs (kept ids in
    slice coordinates, warped scores, count, status).
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
                           repetition_penalty=repetition_penalty, out_capacity=capacity, **kw)


def pack_slice(local, offset, capacity, out=None):
    """This rank's exchange records int32 [rows, 2 * capacity + 2] (the wire format
    of sv_merge_shards): warped scores (float bits), global ids, count, status."""
    R = local["token"].shape[0]
    rec = out if out is not None else torch.empty((R, record_width(capacity)), dtype=torch.int32,
                                                  device=local["token"].device)
    if rec.is_cuda:
        return ops.pack_slice(local, offset, capacity, rec)
    rec[:, :capacity] = local["score"].view(torch.int32)
    rec[:, capacity:2 * capacity] = local["idx"] + offset
    rec[:, 2 * capacity] = local["count"]
    rec[:, 2 * capacity + 1] = local["status"]
    return rec


def all_gather_records(rec, group=None):
    """[world, rows, width] records of every rank (rank order)."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(rec.shape), dtype=rec.dtype, device=rec.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(world * rec.shape[0], rec.shape[1]), rec.contiguous(), group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, rec.contiguous(), group=group)
    return out


def sample_step_vocab_sharded(shard_logits, uniforms, *, offset, seen_bits=None, seen=None, temperature=1.5,
                              top_p=0.9, top_k=50, keep=1, repetition_penalty=3.1, capacity=64, out_capacity=0,
                              group=None, step_fn=None, merge_fn=None, out=None):
    """The vocab-sharded sample step, called by every rank of `group` with its slice.

    Every rank returns the same dict: token int64 [rows], count int32 [rows], status
    int32 [rows] (SV_ST_SHARD_OVERFLOW where a slice's tie group outgrew
    `capacity`: sample that row unsharded), and idx / prob [rows, out_capacity].
    step_fn / merge_fn replace slice_step / ops.merge_shards (the tests use them to
    run the exchange on CPU ranks).
    """
    local = (step_fn or slice_step)(shard_logits, uniforms, offset=offset, seen_bits=seen_bits, seen=seen,
                                    temperature=temperature, top_k=top_k, keep=keep,
                                    repetition_penalty=repetition_penalty, capacity=capacity)
    packed = all_gather_records(pack_slice(local, offset, capacity), group)
    return (merge_fn or ops.merge_shards)(packed, uniforms, capacity=capacity, top_p=top_p, top_k=top_k, keep=keep,
                                          out_capacity=out_capacity, out=out)


def beam_step_vocab_sharded(shard_logits, running_scores, uniforms, *, offset, vocab, seen_bits=None, seen=None,
                            temperature=1.5, top_p=0.9, top_k=50, keep=2, repetition_penalty=3.1, capacity=64,
                            num_picks=None, out_capacity=0, group=None, stats_fn=None, logprob_fn=None,
                            step_fn=None, merge_fn=None, out=None):
    """The vocab-sharded beam step (runtime_shared.py:230-235), called by every rank
    of `group` with its slice [beams, width] of every beam's logits at `offset`.

    Three exchanges: the slices' maxima and NaN / +inf flags (all-reduce MAX), their
    exact fixed-point exp sums against the global maximum (all-reduce SUM, int64),
    then the slices' kept lists (all-gather).  Between them each rank forms its
    slice's log_softmax and runs the slice step on it (penalty, temperature, the
    slice's top-k with ties; top-p off).  Every rank returns beam_step's dict for
    the whole rows (picks are beam * vocab + token).  stats_fn / logprob_fn /
    step_fn / merge_fn replace the CUDA calls (the tests run the exchange on CPU
    ranks with them).
    """
    B = shard_logits.shape[0]
    stats = stats_fn or ops.beam_slice_stats
    first = stats(shard_logits)  # fresh tensors: reduced in place
    gmax, gflags = first["max"], first["flags"]
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(gflags, op=dist.ReduceOp.MAX, group=group)
    gsum = stats(shard_logits, global_max=gmax)["sum"]
    dist.all_reduce(gsum, op=dist.ReduceOp.SUM, group=group)
    lp = (logprob_fn or ops.beam_slice_logprobs)(shard_logits, gmax, gsum)
    dummy = torch.zeros(B, dtype=torch.float32, device=lp.device)
    local = (step_fn or slice_step)(lp, dummy, offset=offset, seen_bits=seen_bits, seen=seen, temperature=temperature,
                                    top_k=top_k, keep=keep, repetition_penalty=repetition_penalty, capacity=capacity)
    packed = all_gather_records(pack_slice(local, offset, capacity), group)
    return (merge_fn or ops.merge_beam_shards)(packed, gmax, gflags, running_scores, uniforms, capacity=capacity,
                                               vocab=vocab, top_p=top_p, top_k=top_k, keep=keep,
                                               num_picks=num_picks, out_capacity=out_capacity, out=out)
