"""The entry points are CUDA-graph capturable (no allocation, sync or host work in
the enqueued path): captured steps replayed on new inputs equal eager calls, as the
reference's CUDA-graph decode (runtime_shared.py:363-386) would replay them."""
import numpy as np
import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
DEV = "cuda"


def capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def test_sample_step_graph_replay(sv):
    g = np.random.default_rng(0)
    R, V = 16, 49152
    x = torch.empty((R, V), device=DEV)
    u = torch.empty(R, device=DEV)
    bits = sv.seen_bitmap(R, V, DEV)
    out = {}
    sv.sample_step(x.normal_(), u.uniform_(), seen_bits=bits, out=out, out_capacity=32)
    graph = capture(lambda: sv.sample_step(x, u, seen_bits=bits, out=out, out_capacity=32))
    for _ in range(3):
        x.copy_(torch.from_numpy((2 * g.standard_normal((R, V))).astype(np.float32)))
        u.copy_(torch.from_numpy(g.random(R).astype(np.float32)))
        bits.copy_(torch.from_numpy(g.integers(-2**31, 2**31 - 1, bits.shape, dtype=np.int64).astype(np.int32)))
        graph.replay()
        eager = sv.sample_step(x, u, seen_bits=bits, out_capacity=32)
        torch.cuda.synchronize()
        for k in ("token", "count", "idx", "prob"):
            assert torch.equal(out[k], eager[k]), k


def test_beam_step_graph_replay(sv):
    d = bench.cfg2()
    x, rs, u, h = (torch.from_numpy(d[k]).to(DEV) for k in ("logits", "running", "uniforms", "history"))
    out = {}
    ws = torch.zeros(sv._lib.lib().sv_beam_workspace_bytes(2, 49152), dtype=torch.uint8, device=DEV)
    sv.beam_step(x, rs, u, history=h, out=out, workspace=ws)
    graph = capture(lambda: sv.beam_step(x, rs, u, history=h, out=out, workspace=ws))
    g = np.random.default_rng(1)
    for _ in range(4):
        x.copy_(torch.from_numpy((2 * g.standard_normal(x.shape)).astype(np.float32)))
        u.copy_(torch.from_numpy(g.random(4).astype(np.float32)))
        graph.replay()
        eager = sv.beam_step(x, rs, u, history=h)
        torch.cuda.synchronize()
        for k in ("picks", "scores", "n", "status"):
            assert torch.equal(out[k], eager[k]), k


def test_loop_guard_graph_replay(sv):
    t = torch.from_numpy(bench.cfg5_tokens(rows=32, length=4096)).to(DEV)
    v = torch.empty(32, dtype=torch.uint8, device=DEV)
    lens = torch.full((32,), 4096, dtype=torch.int32, device=DEV)
    graph = capture(lambda: sv.loop_guard(t, lens, out=v))
    graph.replay()
    torch.cuda.synchronize()
    assert v.bool().tolist() == sv.loop_guard(t, lens).tolist()
