"""The vocab-sharded sample step across GPUs: one process per GPU, NCCL all-gather.

Runs only on a box with at least 2 GPUs (skipped otherwise).  Each rank holds one
slice of the vocabulary; every rank's merged tokens, kept sets and probabilities
must equal the oracle on the whole row.  The process group has a short timeout, so
a rank that fails ends the others' collective with an error rather than a wait.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
ROWS, V, CAP = 64, 49152, 64


def _data():
    g = np.random.default_rng(41)
    x = (2 * g.standard_normal((ROWS, V))).astype(np.float32)
    seen = np.zeros((ROWS, V), bool)
    seen[np.arange(ROWS)[:, None], g.integers(0, V, (ROWS, 4096))] = True
    u = g.random(ROWS).astype(np.float32)
    return x, seen, u


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        import __graft_entry__
        sv = __graft_entry__.load_package()
        x, seen, u = _data()
        w = V // world
        off = rank * w
        packed = np.packbits(seen, axis=1, bitorder="little")
        bits = torch.from_numpy(np.ascontiguousarray(packed).view(np.int32)).to(dev)
        out = sv.sharded.sample_step_vocab_sharded(
            torch.from_numpy(np.ascontiguousarray(x[:, off:off + w])).to(dev), torch.from_numpy(u).to(dev),
            offset=off, seen_bits=bits, capacity=CAP, out_capacity=CAP)
        torch.cuda.synchronize()
        q.put((rank, {k: v.cpu().numpy() for k, v in out.items()}))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_vocab_sharded_across_gpus():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x, seen, u = _data()
    ref = O.sample(x, u, seen=seen.astype(np.uint8), temperature=1.5, top_p=0.9, top_k=50, keep=1, cap=CAP)
    for rank in range(world):
        g = got[rank]
        np.testing.assert_array_equal(g["status"], ref["status"])
        np.testing.assert_array_equal(g["token"], ref["token"])
        np.testing.assert_array_equal(g["count"], ref["count"])
        for r in range(ROWS):
            n = min(int(ref["count"][r]), CAP)
            np.testing.assert_array_equal(g["idx"][r, :n], ref["idx"][r, :n])
            np.testing.assert_array_equal(g["prob"][r, :n], ref["prob"][r, :n])
