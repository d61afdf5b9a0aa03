"""The vocab-sharded sample and beam steps across GPUs: one process per GPU, NCCL.

Runs on every GPU of the box (up to 8; on a one-GPU box a single rank holds the
whole vocabulary).  Each rank holds one slice of the vocabulary and runs the step
eagerly, then as one captured CUDA graph (slice kernels, NCCL collectives, merge)
replayed twice with new uniforms written in place; every rank's merged tokens,
kept sets and probabilities must equal the oracle on the whole row.  The process
group has a short timeout, so a rank that fails ends the others' collective with an
error rather than a wait; graphs are released before the group is destroyed.
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
    sampler = None
    try:
        import __graft_entry__
        sv = __graft_entry__.load_package()
        x, seen, u = _data()
        off, w, stride = sv.sharded.slice_bounds(V, rank, world)
        packed = np.packbits(seen, axis=1, bitorder="little")
        bits = torch.from_numpy(np.ascontiguousarray(packed).view(np.int32)).to(dev)
        xs = torch.from_numpy(np.ascontiguousarray(x[:, off:off + w])).to(dev)
        us = torch.from_numpy(u).to(dev)
        res = {}
        out = sv.sharded.sample_step_vocab_sharded(xs, us, offset=off, slice_stride=stride, seen_bits=bits,
                                                   capacity=CAP, out_capacity=CAP)
        res["eager"] = {k: v.cpu().numpy() for k, v in out.items()}
        sampler = sv.sharded.VocabShardedSampler(xs, us, offset=off, slice_stride=stride, seen_bits=bits,
                                                 capacity=CAP, out_capacity=CAP).capture()
        for n, uu in enumerate((u, _uniforms2())):
            us.copy_(torch.from_numpy(uu))
            out = sampler()
            torch.cuda.synchronize()
            res[f"graph{n}"] = {k: v.cpu().numpy() for k, v in out.items()}
        q.put((rank, res))
    finally:
        if sampler is not None:
            sampler.release()
        dist.destroy_process_group()


def _uniforms2():
    return np.random.default_rng(42).random(ROWS).astype(np.float32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check_sample(g, ref):
    np.testing.assert_array_equal(g["status"], ref["status"])
    np.testing.assert_array_equal(g["token"], ref["token"])
    np.testing.assert_array_equal(g["count"], ref["count"])
    for r in range(ROWS):
        n = min(int(ref["count"][r]), CAP)
        np.testing.assert_array_equal(g["idx"][r, :n], ref["idx"][r, :n])
        np.testing.assert_array_equal(g["prob"][r, :n], ref["prob"][r, :n])


def _run(target, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


def test_vocab_sharded_across_gpus():
    world = min(torch.cuda.device_count(), 8)
    got = _run(_worker, world)
    x, seen, u = _data()
    kw = dict(seen=seen.astype(np.uint8), temperature=1.5, top_p=0.9, top_k=50, keep=1, cap=CAP)
    ref = O.sample(x, u, **kw)
    ref2 = O.sample(x, _uniforms2(), **kw)
    for rank in range(world):
        _check_sample(got[rank]["eager"], ref)
        _check_sample(got[rank]["graph0"], ref)
        _check_sample(got[rank]["graph1"], ref2)


BEAMS = 4


def _beam_data():
    g = np.random.default_rng(43)
    x = (2.5 * g.standard_normal((BEAMS, V))).astype(np.float32)
    seen = np.zeros((BEAMS, V), bool)
    seen[np.arange(BEAMS)[:, None], g.integers(0, V, (BEAMS, 2048))] = True
    running = np.array([-1.0, -4.0, -2.5, -30.0], np.float32)
    u = g.random(2 * BEAMS).astype(np.float32)
    return x, seen, running, u


def _beam_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    step = None
    try:
        import __graft_entry__
        sv = __graft_entry__.load_package()
        x, seen, running, u = _beam_data()
        off, w, stride = sv.sharded.slice_bounds(V, rank, world)
        packed = np.packbits(seen, axis=1, bitorder="little")
        bits = torch.from_numpy(np.ascontiguousarray(packed).view(np.int32)).to(dev)
        xs = torch.from_numpy(np.ascontiguousarray(x[:, off:off + w])).to(dev)
        rs = torch.from_numpy(running).to(dev)
        us = torch.from_numpy(u).to(dev)
        res = {}
        out = sv.sharded.beam_step_vocab_sharded(xs, rs, us, offset=off, vocab=V, slice_stride=stride,
                                                 seen_bits=bits, capacity=CAP, out_capacity=CAP)
        res["eager"] = {k: v.cpu().numpy() for k, v in out.items()}
        for method in ("exchange", "gather"):
            step = sv.sharded.VocabShardedBeamStep(xs, rs, us, offset=off, vocab=V, slice_stride=stride,
                                                   seen_bits=bits, capacity=CAP, out_capacity=CAP,
                                                   method=method).capture()
            for n, uu in enumerate((u, _beam_uniforms2())):
                us.copy_(torch.from_numpy(uu))
                out = step()
                torch.cuda.synchronize()
                res[f"{method}{n}"] = {k: v.cpu().numpy() for k, v in out.items()}
            step.release()
            step = None
        q.put((rank, res))
    finally:
        if step is not None:
            step.release()
        dist.destroy_process_group()


def _beam_uniforms2():
    return np.random.default_rng(44).random(2 * BEAMS).astype(np.float32)


def _check_beam(g, ref):
    assert int(g["status"][0]) == ref["status"] == 0
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


def test_vocab_sharded_beam_step_across_gpus():
    """The beam step with every beam's vocabulary split across the GPUs: two
    all-reduces (the log_softmax statistics) and one all-gather of the kept lists,
    or one all-gather of the slices and the whole-row beam kernel."""
    world = min(torch.cuda.device_count(), 8)
    got = _run(_beam_worker, world)
    x, seen, running, u = _beam_data()
    kw = dict(seen=seen.astype(np.uint8), temperature=1.5, top_p=0.9, top_k=50, keep=2, npick=2 * BEAMS)
    ref = O.beam(x, running, u, **kw)
    ref2 = O.beam(x, running, _beam_uniforms2(), **kw)
    for rank in range(world):
        _check_beam(got[rank]["eager"], ref)
        for method in ("exchange", "gather"):
            _check_beam(got[rank][f"{method}0"], ref)
            _check_beam(got[rank][f"{method}1"], ref2)
