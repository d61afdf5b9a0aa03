"""GPU parity of the vocab-sharded beam step, slices emulated on one GPU.

Each slice runs the rank-side calls of sharded.beam_step_vocab_sharded:
- its statistics (sv_beam_slice_stats), reduced across the slices as the all-reduces
  would (MAX of maxima and flags, SUM of the int64 exp sums);
- its log_softmax (sv_beam_slice_logprobs) and slice step;
- its exchange block written by the slice step (sv_merge_beam_slices' layout)
  or packed records (sv_pack_slice, for sv_merge_beam_shards), stacked as an
  all-gather lays them out, then the merge.

Picks, picked scores, pick count, status and the per-beam kept lists must equal the
oracle's beam step on the whole rows, bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bitmap(seen):
    b = np.packbits(seen.astype(bool), axis=1, bitorder="little")
    b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int32)).to(DEV)


def run_sharded(sv, x, seen, running, u, shards, cap, dtype=torch.float32, T=1.5, p=0.9, top_k=50, out_cap=128,
                layout="blocks"):
    B, V = x.shape
    xd = torch.from_numpy(x).to(DEV).to(dtype)
    rs = torch.from_numpy(running).to(DEV)
    ud = torch.from_numpy(u).to(DEV)
    bits = bitmap(seen)
    w = V // shards
    sl = [xd[:, s * w:(s + 1) * w] for s in range(shards)]
    first = [sv.ops.beam_slice_stats(t) for t in sl]
    gmax = torch.stack([f["max"] for f in first]).amax(0).contiguous()
    gflags = torch.stack([f["flags"] for f in first]).amax(0).contiguous()
    gsum = torch.stack([sv.ops.beam_slice_stats(t, global_max=gmax)["sum"] for t in sl]).sum(0).contiguous()
    parts = []
    dummy = torch.zeros(B, dtype=torch.float32, device=DEV)
    for s, t in enumerate(sl):
        lp = sv.ops.beam_slice_logprobs(t, gmax, gsum)
        kw = dict(offset=s * w, seen_bits=bits, temperature=T, top_k=top_k, keep=2, capacity=cap)
        if layout == "blocks":
            blk = torch.empty(sv.ops.block_len(B, cap), dtype=torch.int32, device=DEV)
            sv.sharded.slice_step(lp, dummy, out=sv.ops.slice_block_outputs(blk, B, cap), **kw)
            parts.append(blk)
        else:
            loc = sv.sharded.slice_step(lp, dummy, **kw)
            rec = torch.empty((B, 2 * cap + 2), dtype=torch.int32, device=DEV)
            parts.append(sv.ops.pack_slice(loc, s * w, cap, rec))
    packed = torch.stack(parts).contiguous()
    extra = dict(beams=B, slice_stride=w) if layout == "blocks" else {}
    out = sv.ops.merge_beam_shards(packed, gmax, gflags, rs, ud, capacity=cap, vocab=V, top_p=p, top_k=top_k,
                                   keep=2, out_capacity=out_cap, **extra)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}, xd.float().cpu().numpy()


def check(got, ref):
    assert int(got["status"][0]) == ref["status"]
    if ref["status"]:
        assert int(got["n"][0]) == 0
        return
    n = int(got["n"][0])
    assert n == ref["n"]
    np.testing.assert_array_equal(got["picks"][:n], ref["picks"])
    np.testing.assert_array_equal(got["scores"][:n], ref["scores"])
    cap = got["kept_idx"].shape[1]
    V = ref["logp"].shape[1]
    for b in range(got["kept_count"].shape[0]):
        ki = np.nonzero(np.isfinite(ref["logp"][b]))[0]
        assert got["kept_count"][b] == len(ki)
        k = min(len(ki), cap)
        np.testing.assert_array_equal(got["kept_idx"][b, :k], ki[:k])
        np.testing.assert_array_equal(got["kept_logprob"][b, :k], ref["logp"][b][ki[:k]])
        np.testing.assert_array_equal(got["kept_prob"][b, :k], ref["probs"][b * V + ki[:k]])


def oracle_beam(xf, seen, running, u, T=1.5, p=0.9, top_k=50):
    return O.beam(xf, running, u, seen=seen, temperature=T, top_p=p, top_k=top_k, keep=2, npick=len(u))


@pytest.mark.parametrize("layout", ["blocks", "records"])
@pytest.mark.parametrize("beams,dtype,shards", [(2, torch.float32, 8), (8, torch.bfloat16, 8), (3, torch.float16, 4),
                                                (1, torch.float32, 2)])
def test_slices_match_whole_rows(sv, beams, dtype, shards, layout):
    """Config 2 / 3 shapes (V = 49152) split into slices of 6144 or more."""
    g = np.random.default_rng(40 + beams)
    x = (2.5 * g.standard_normal((beams, 49152))).astype(np.float32)
    x[:, g.choice(49152, 400, replace=False)] += 5.0
    seen = np.zeros(x.shape, np.uint8)
    np.put_along_axis(seen, g.integers(0, 49152, (beams, 3000)), 1, axis=1)
    running = np.sort(g.uniform(-60, 0, beams)).astype(np.float32)[::-1].copy()
    u = g.random(2 * beams).astype(np.float32)
    got, xf = run_sharded(sv, x, seen, running, u, shards, cap=64, dtype=dtype, layout=layout)
    check(got, oracle_beam(xf, seen, running, u))


@pytest.mark.parametrize("case", ["nan", "posinf", "allneginf", "one_slice_empty", "running_behind"])
def test_statuses_and_edges(sv, case):
    """The log_softmax stage's statuses come from the reduced statistics (a NaN or
    +inf in any slice, no finite logit anywhere); a slice without a finite logit
    contributes nothing; a beam far behind draws nothing."""
    g = np.random.default_rng(7)
    x = (2 * g.standard_normal((2, 8192))).astype(np.float32)
    running = np.array([0.0, -5.0], np.float32)
    if case == "nan":
        x[1, 7000] = np.nan
    elif case == "posinf":
        x[0, 100] = np.inf
    elif case == "allneginf":
        x[:] = -np.inf
    elif case == "one_slice_empty":
        x[:, 2048:4096] = -np.inf
    else:
        running = np.array([0.0, -1e9], np.float32)
    seen = (g.random(x.shape) < 0.02).astype(np.uint8)
    u = g.random(4).astype(np.float32)
    got, xf = run_sharded(sv, x, seen, running, u, shards=4, cap=64)
    check(got, oracle_beam(xf, seen, running, u))


def test_agrees_with_unsharded_beam_step(sv):
    """The same inputs through sv_beam_step on the whole rows."""
    g = np.random.default_rng(9)
    x = (2 * g.standard_normal((4, 16384))).astype(np.float32)
    seen = (g.random(x.shape) < 0.03).astype(np.uint8)
    running = np.array([-3.0, -1.0, -8.0, -2.0], np.float32)
    u = g.random(8).astype(np.float32)
    got, _ = run_sharded(sv, x, seen, running, u, shards=4, cap=64)
    whole = sv.beam_step(torch.from_numpy(x).to(DEV), torch.from_numpy(running).to(DEV), torch.from_numpy(u).to(DEV),
                         seen_bits=bitmap(seen), out_capacity=128)
    torch.cuda.synchronize()
    n = int(whole["n"].item())
    assert int(got["n"][0]) == n
    np.testing.assert_array_equal(got["picks"][:n], whole["picks"][:n].cpu().numpy())
    np.testing.assert_array_equal(got["scores"][:n], whole["scores"][:n].cpu().numpy())
