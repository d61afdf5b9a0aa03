"""Host side of the multi-GPU paths, on CPU ranks (gloo, world size 2).

The vocab-sharded step runs its real host pipeline (slicing of the logits and the
seen mask, the exchange records, the all-gather, the merge's input layout) with
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


def oracle_merge(packed, uniforms, *, capacity, top_p, top_k, keep, out_capacity, out=None):
    p = packed.numpy()
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
