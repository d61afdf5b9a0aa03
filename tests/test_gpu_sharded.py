"""GPU parity of the vocab-sharded sample step, slices emulated on one GPU.

Each slice runs sharded.slice_step (sv_sample_step with top_p = 1 and a kept-list
capacity) on its view of the logits and of the seen bitmap, writing its exchange
block directly (sv_merge_slices' layout) or packing records (sv_pack_slice, for
sv_merge_shards); the blocks or records are stacked as an all-gather lays them out
and merged.  The result must equal the oracle on the whole row, bit for bit
(tokens, kept sets, probabilities, statuses).
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


def run_sharded(sv, x, seen, u, shards, cap, T=1.5, p=0.9, top_k=50, keep=1, out_cap=64, layout="blocks"):
    xd = torch.from_numpy(x).to(DEV)
    ud = torch.from_numpy(u).to(DEV)
    bits = bitmap(seen)
    R = x.shape[0]
    w = x.shape[1] // shards
    parts = []
    for s in range(shards):
        kw = dict(offset=s * w, seen_bits=bits, temperature=T, top_k=top_k, keep=keep, capacity=cap)
        if layout == "blocks":
            blk = torch.empty(sv.ops.block_len(R, cap), dtype=torch.int32, device=DEV)
            sv.sharded.slice_step(xd[:, s * w:(s + 1) * w], ud, out=sv.ops.slice_block_outputs(blk, R, cap), **kw)
            parts.append(blk)
        else:
            loc = sv.sharded.slice_step(xd[:, s * w:(s + 1) * w], ud, **kw)
            rec = torch.empty((R, 2 * cap + 2), dtype=torch.int32, device=DEV)
            parts.append(sv.ops.pack_slice(loc, s * w, cap, rec))
    packed = torch.stack(parts).contiguous()
    if layout == "blocks":
        out = sv.merge_shards(packed, ud, capacity=cap, top_p=p, top_k=top_k, keep=keep, out_capacity=out_cap,
                              rows=R, slice_stride=w)
    else:
        out = sv.merge_shards(packed, ud, capacity=cap, top_p=p, top_k=top_k, keep=keep, out_capacity=out_cap)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


def check(got, ref, cap):
    np.testing.assert_array_equal(got["status"], ref["status"])
    np.testing.assert_array_equal(got["token"], ref["token"])
    np.testing.assert_array_equal(got["count"], ref["count"])
    for r in range(len(got["token"])):
        n = min(int(ref["count"][r]), cap)
        np.testing.assert_array_equal(got["idx"][r, :n], ref["idx"][r, :n])
        np.testing.assert_array_equal(got["prob"][r, :n], ref["prob"][r, :n])


@pytest.mark.parametrize("layout", ["blocks", "records"])
@pytest.mark.parametrize("hist", [2048, 16384])
def test_cfg5_eight_slices_match_whole_row(sv, hist, layout):
    """Config 5's split: V=49152 in 8 slices of 6144, top-50 lists, 256 rows."""
    g = np.random.default_rng(31)
    x = (2 * g.standard_normal((256, 49152))).astype(np.float32)
    seen = np.zeros(x.shape, np.uint8)
    ids = g.integers(0, 49152, (256, hist))
    np.put_along_axis(seen, ids, 1, axis=1)
    u = g.random(256).astype(np.float32)
    got = run_sharded(sv, x, seen, u, shards=8, cap=64, layout=layout)
    ref = O.sample(x, u, seen=seen, temperature=1.5, top_p=0.9, top_k=50, keep=1, cap=64)
    check(got, ref, 64)


@pytest.mark.parametrize("layout", ["blocks", "records"])
@pytest.mark.parametrize("T,p,keep", [(1.0, 1.0, 1), (0.7, 0.5, 3), (1.5, 0.95, 2)])
def test_settings_and_special_rows(sv, T, p, keep, layout):
    g = np.random.default_rng(32)
    x = (2 * g.standard_normal((6, 8192))).astype(np.float32)
    x[1, 5000] = np.nan
    x[2, 4096:] = -np.inf
    x[3, :] = -np.inf
    x[4, 10:30] = 9.0   # a tie group at the top of slice 0
    x[5, 8000] = np.inf
    seen = (g.random(x.shape) < 0.05).astype(np.uint8)
    u = g.random(6).astype(np.float32)
    got = run_sharded(sv, x, seen, u, shards=4, cap=64, T=T, p=p, keep=keep, layout=layout)
    ref = O.sample(x, u, seen=seen, temperature=T, top_p=p, top_k=50, keep=keep, cap=64)
    assert ref["status"].tolist() == [0, 1, 0, 3, 0, 2]
    check(got, ref, 64)


def test_tie_overflow_is_reported(sv):
    """A slice whose tie group at its k-th largest outgrows the list capacity."""
    x = np.zeros((2, 4096), np.float32)
    x[1] = np.random.default_rng(33).standard_normal(4096).astype(np.float32)
    u = np.array([0.3, 0.6], np.float32)
    got = run_sharded(sv, x, np.zeros(x.shape, np.uint8), u, shards=2, cap=64)
    assert got["status"].tolist() == [6, 0]
    assert got["token"][0] == -1
