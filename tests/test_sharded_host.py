"""Host side of the multi-GPU paths, on CPU ranks (gloo, world size 2).

The vocab-sharded step runs its real host pipeline (slicing of the logits and the
seen mask, the exchange blocks, the all-gather, the merge's input layout) with
the CUDA kernels replaced by the oracle: the per-slice step is oracle.sample on the
slice with top_p = 1, and the merge is oracle.sample, with temperature 1 and no
penalty, on a row that holds only the gathered candidates (their warped scores at
their global ids, -inf elsewhere).  Its tokens, kept sets and probabilities must
equal oracle.sample on the whole row: the union of the slices' top-k lists holds
the row's whole top-k set.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

R, V, CAP, WORLD = 6, 4096, 64, 2


def _data():
    g = np.random.default_rng(21)
    x = (2 * g.standard_normal((R, V))).astype(np.float32)
    x[1, 3000] = np.nan                      # a NaN in rank 1's slice
    x[2, 2048:] = -np.inf                    # rank 1's slice has no finite logit
    x[3, :2048] = -np.inf                    # rank 0's slice has none
    x[4, 100:120] = 9.0                      # a tie group at the top, in rank 0's slice
    seen = (g.random((R, V)) < 0.05).astype(np.uint8)
    u = g.random(R).astype(np.float32)
    return x, seen, u


def oracle_step(shard_logits, uniforms, *, offset, seen_bits=None, seen=None, temperature, top_k, keep,
                repetition_penalty, capacity):
    x = shard_logits.numpy()
    w = x.shape[1]
    s = None if seen is None else seen[:, offset:offset + w].numpy()
    r = O.sample(x, uniforms.numpy(), seen=s, temperature=temperature, top_p=1.0, top_k=top_k, keep=keep,
                 rep_penalty=repetition_penalty, cap=capacity, dense=True)
    score = np.take_along_axis(r["scores"], np.clip(r["idx"], 0, w - 1), axis=1)
    return {"token": torch.from_numpy(r["token"]), "count": torch.from_numpy(r["count"]),
            "status": torch.from_numpy(r["status"]), "idx": torch.from_numpy(r["idx"]),
            "score": torch.from_numpy(np.ascontiguousarray(score, np.float32))}


def records(blocks, rows, capacity, slice_stride):
    """The all-gathered exchange blocks [shards, block_len] as per-shard records
    [shards, rows, 2 * capacity + 2] with global ids (the layout the merge reads)."""
    b = blocks.numpy()
    S, RC = b.shape[0], rows * capacity
    out = np.zeros((S, rows, 2 * capacity + 2), np.int32)
    for s in range(S):
        out[s, :, :capacity] = b[s, :RC].reshape(rows, capacity)
        out[s, :, capacity:2 * capacity] = b[s, RC:2 * RC].reshape(rows, capacity) + s * slice_stride
        out[s, :, 2 * capacity] = b[s, 2 * RC:2 * RC + rows]
        out[s, :, 2 * capacity + 1] = b[s, 2 * RC + rows:]
    return out


def oracle_merge(blocks, uniforms, *, capacity, top_p, top_k, keep, out_capacity, out=None, rows, slice_stride):
    p = records(blocks, rows, capacity, slice_stride)
    S, Rr, _ = p.shape
    sparse = np.full((Rr, V), -np.inf, np.float32)
    bad = np.zeros(Rr, np.int32)
    for r in range(Rr):
        err = 0
        for s in range(S):
            cnt, st = p[s, r, 2 * capacity], p[s, r, 2 * capacity + 1]
            if st == 3:
                continue
            if st:
                err |= 1 << int(st)
                continue
            take = min(int(cnt), capacity)
            sparse[r, p[s, r, capacity:capacity + take]] = p[s, r, :take].view(np.float32)
        bad[r] = next((b for b in range(1, 8) if err >> b & 1), 0)
    res = O.sample(sparse, uniforms.numpy(), temperature=1.0, top_p=top_p, top_k=top_k, keep=keep,
                   cap=out_capacity)
    res["status"] = np.where(bad > 0, bad, res["status"]).astype(np.int32)
    res["token"] = np.where(bad > 0, -1, res["token"])
    res["count"] = np.where(bad > 0, 0, res["count"]).astype(np.int32)
    return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in res.items()}


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        import __graft_entry__
        sv = __graft_entry__.load_package()
        x, seen, u = _data()
        w = V // WORLD
        off = rank * w
        res = sv.sharded.sample_step_vocab_sharded(
            torch.from_numpy(np.ascontiguousarray(x[:, off:off + w])), torch.from_numpy(u), offset=off,
            seen=torch.from_numpy(seen), temperature=1.5, top_p=0.9, top_k=50, keep=1, capacity=CAP,
            out_capacity=CAP, step_fn=oracle_step, merge_fn=oracle_merge)
        q.put((rank, {k: v.numpy() for k, v in res.items()}))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_vocab_sharded_exchange_matches_whole_row():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, seen, u = _data()
    ref = O.sample(x, u, seen=seen, temperature=1.5, top_p=0.9, top_k=50, keep=1, cap=CAP)
    assert ref["status"].tolist() == [0, 1, 0, 0, 0, 0]
    for rank in range(WORLD):
        g = got[rank]
        np.testing.assert_array_equal(g["status"], ref["status"])
        np.testing.assert_array_equal(g["token"], ref["token"])
        np.testing.assert_array_equal(g["count"], ref["count"])
        for r in range(R):
            n = min(int(ref["count"][r]), CAP)
            np.testing.assert_array_equal(g["idx"][r, :n], ref["idx"][r, :n])
            np.testing.assert_array_equal(g["prob"][r, :n], ref["prob"][r, :n])


@pytest.mark.parametrize("rows,world", [(1024, 1), (1024, 2), (1024, 8), (5, 8), (7, 3)])
def test_row_blocks_cover_rows_once(rows, world):
    import __graft_entry__
    sv = __graft_entry__.load_package()
    seen = []
    for rank in range(world):
        lo, hi = sv.sharded.row_block(rows, rank, world)
        seen.extend(range(lo, hi))
    assert seen == list(range(rows))


# ----------------------------------------------------------- vocab-sharded beam step

BEAMS = 4


def _beam_data():
    g = np.random.default_rng(23)
    x = (2.5 * g.standard_normal((BEAMS, V))).astype(np.float32)
    x[2, 2048:] = -np.inf                    # rank 1's slice of beam 2 has no finite logit
    seen = (g.random((BEAMS, V)) < 0.05).astype(np.uint8)
    running = np.array([-1.0, -3.0, -0.5, -12.0], np.float32)
    u = g.random(2 * BEAMS).astype(np.float32)
    return x, seen, running, u


def _fixw(w):
    return (np.asarray(w, np.float32) * np.float32(2.0 ** 44)).astype(np.uint64)


def oracle_stats(shard_logits, global_max=None):
    """sv_beam_slice_stats restated on the host with the oracle's exp."""
    x = shard_logits.numpy()
    if global_max is None:
        flags = np.where(np.isnan(x).any(1), 2, np.where(np.isposinf(x).any(1), 1, 0)).astype(np.int32)
        return {"max": torch.from_numpy(np.max(x, axis=1).astype(np.float32)), "flags": torch.from_numpy(flags)}
    M = global_max.numpy()
    sums = np.zeros(len(M), np.uint64)
    for b in range(len(M)):
        if np.isfinite(M[b]):
            sums[b] = _fixw(O.exp(x[b] - M[b])).sum(dtype=np.uint64)
    return {"sum": torch.from_numpy(sums.view(np.int64))}


def oracle_logprobs(shard_logits, gmax, gsum):
    x = shard_logits.numpy()
    M = gmax.numpy()
    L = O.log_fixed(gsum.numpy().view(np.uint64)).astype(np.float32)
    return torch.from_numpy(((x - M[:, None]).astype(np.float32) - L[:, None]).astype(np.float32))


def oracle_beam_merge(blocks, gmax, gflags, running, uniforms, *, capacity, vocab, top_p, top_k, keep, num_picks,
                      out_capacity, out=None, beams, slice_stride):
    """sv_merge_beam_shards restated on the host: each beam's kept list from the
    union (oracle.sample, temperature 1, on a row holding only the gathered warped
    log-probs), then the flattened softmax and the draws as oracle.beam makes them."""
    p = records(blocks, beams, capacity, slice_stride)
    S, B, _ = p.shape
    fl, M, rs, u = gflags.numpy(), gmax.numpy(), running.numpy(), uniforms.numpy()
    sparse = np.full((B, vocab), -np.inf, np.float32)
    status = np.zeros(B, np.int32)
    for b in range(B):
        err = 0
        for s in range(S):
            cnt, st = p[s, b, 2 * capacity], p[s, b, 2 * capacity + 1]
            if st == 3:
                continue
            if st:
                err |= 1 << int(st)
                continue
            take = min(int(cnt), capacity)
            sparse[b, p[s, b, capacity:capacity + take]] = p[s, b, :take].view(np.float32)
        status[b] = 1 if fl[b] >= 2 else 2 if fl[b] == 1 else 3 if M[b] == -np.inf else \
            next((e for e in range(1, 8) if err >> e & 1), 0)
    kept = O.sample(sparse, np.zeros(B, np.float32), temperature=1.0, top_p=top_p, top_k=top_k, keep=keep,
                    cap=vocab)
    P = num_picks or 2 * B
    res = {"picks": np.full(P, -1, np.int64), "scores": np.zeros(P, np.float32), "n": np.zeros(1, np.int32),
           "status": np.zeros(1, np.int32), "kept_count": np.zeros(B, np.int32),
           "kept_idx": np.full((B, out_capacity), -1, np.int32),
           "kept_logprob": np.zeros((B, out_capacity), np.float32)}
    flat_i, flat_s = [], []
    for b in range(B):
        n_b = int(kept["count"][b]) if status[b] == 0 else 0
        ids = kept["idx"][b, :n_b]
        res["kept_count"][b] = n_b
        k = min(n_b, out_capacity)
        res["kept_idx"][b, :k] = ids[:k]
        res["kept_logprob"][b, :k] = sparse[b, ids[:k]]
        flat_i += [b * vocab + int(i) for i in ids]
        flat_s += [np.float32(sparse[b, i]) + rs[b] for i in ids]
    bad = [int(st) for st in status if st]
    if bad or not flat_s:
        res["status"][0] = bad[0] if bad else 3
        return {k: torch.from_numpy(v) for k, v in res.items()}
    sc = np.asarray(flat_s, np.float32)
    Ms = sc.max()
    ex = O.exp(sc - Ms)
    W = _fixw(ex)
    Sf = np.float32(np.float32(W.sum(dtype=np.uint64)) * np.float32(2.0 ** -44))
    prob = (ex / Sf).astype(np.float32)
    rem = prob > 0
    n = min(P, int(rem.sum()))
    for j in range(n):
        TW = int(W[rem].sum(dtype=np.uint64))
        if TW > 0:
            t = int(O.mulfloor(np.array([TW], np.uint64), np.array([u[j]], np.float32))[0])
            c, pick = 0, -1
            for f in np.nonzero(rem)[0]:
                c += int(W[f])
                if c > t:
                    pick = f
                    break
        else:
            cand = np.nonzero(rem)[0]
            pick = cand[np.argmax(prob[cand])]
        rem[pick] = False
        res["picks"][j] = flat_i[pick]
        res["scores"][j] = sc[pick]
    res["n"][0] = n
    return {k: torch.from_numpy(v) for k, v in res.items()}


def _beam_worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        import __graft_entry__
        sv = __graft_entry__.load_package()
        x, seen, running, u = _beam_data()
        w = V // WORLD
        off = rank * w
        res = sv.sharded.beam_step_vocab_sharded(
            torch.from_numpy(np.ascontiguousarray(x[:, off:off + w])), torch.from_numpy(running),
            torch.from_numpy(u), offset=off, vocab=V, seen=torch.from_numpy(seen), capacity=CAP, out_capacity=CAP,
            stats_fn=oracle_stats, logprob_fn=oracle_logprobs, step_fn=oracle_step, merge_fn=oracle_beam_merge)
        q.put((rank, {k: v.numpy() for k, v in res.items()}))
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_beam_exchange_matches_whole_rows():
    """The sharded beam step's host pipeline (two all-reduces, one all-gather) on
    two CPU ranks, with the CUDA calls replaced by oracle restatements: every rank's
    picks, scores and kept lists equal oracle.beam on the whole rows."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_beam_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, seen, running, u = _beam_data()
    ref = O.beam(x, running, u, seen=seen, temperature=1.5, top_p=0.9, top_k=50, keep=2, npick=2 * BEAMS)
    assert ref["status"] == 0
    for rank in range(WORLD):
        g = got[rank]
        assert int(g["status"][0]) == 0
        n = int(g["n"][0])
        assert n == ref["n"]
        np.testing.assert_array_equal(g["picks"][:n], ref["picks"])
        np.testing.assert_array_equal(g["scores"][:n], ref["scores"])
        for b in range(BEAMS):
            ki = np.nonzero(np.isfinite(ref["logp"][b]))[0]
            assert g["kept_count"][b] == len(ki)
            k = min(len(ki), CAP)
            np.testing.assert_array_equal(g["kept_idx"][b, :k], ki[:k])
            np.testing.assert_array_equal(g["kept_logprob"][b, :k], ref["logp"][b][ki[:k]])
