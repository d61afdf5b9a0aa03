"""GPU parity of the loop-guard kernel (runtime_shared.py:156-167) against the
oracle and the reference's golden verdicts, through the C ABI (sv_loop_guard)."""
import numpy as np
import pytest
import torch

import bench
from _golden import GOLDEN, cfg5_fixture
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_golden_verdicts(sv, dtype):
    d = np.load(GOLDEN + "/repeat.npz")
    t = torch.from_numpy(d["tokens"]).to(DEV).to(dtype)
    v = sv.loop_guard(t, torch.from_numpy(d["lengths"]).to(DEV))
    np.testing.assert_array_equal(v.cpu().numpy(), d["verdict"])


def test_cfg5_full_size_verdicts(sv):
    t = bench.cfg5_tokens()
    v = sv.loop_guard(torch.from_numpy(t).to(DEV))
    ref = O.repeating(t)
    np.testing.assert_array_equal(v.cpu().numpy(), ref)
    assert ref[:128].all() and not ref[128:].any()


def test_cfg5_reference_verdicts(sv):
    """Config 5 at full size against the reference's own _repeating verdicts."""
    t, verdict = cfg5_fixture()
    v = sv.loop_guard(torch.from_numpy(t).to(DEV))
    np.testing.assert_array_equal(v.cpu().numpy(), verdict)


@pytest.mark.parametrize("window,repeats", [(1, 3), (8, 2), (64, 3), (64, 5), (200, 3), (1024, 2)])
def test_windows_repeats_and_ragged_lengths(sv, window, repeats):
    g = np.random.default_rng(window * 10 + repeats)
    R, L = 24, 6000
    t = g.integers(0, 5, (R, L)).astype(np.int32)  # tiny alphabet: many hash-equal starts
    lengths = g.integers(0, L + 1, R).astype(np.int32)
    lengths[:3] = [0, window * repeats - 1, window * repeats]
    for r in range(0, R, 3):
        n = lengths[r]
        if n >= window:
            w = t[r, n - window:n].copy()
            for k in range(1, repeats):
                s = n - window - k * (window + 7)
                if s >= 0:
                    t[r, s:s + window] = w
    v = sv.loop_guard(torch.from_numpy(t).to(DEV), torch.from_numpy(lengths).to(DEV), window=window,
                      repeats=repeats)
    np.testing.assert_array_equal(v.cpu().numpy(), O.repeating(t, lengths, window, repeats))


def test_all_equal_and_periodic(sv):
    t = np.ones((3, 5000), np.int32)
    t[1] = np.arange(5000) % 65        # period 65: windows repeat every 65 tokens
    t[2] = np.arange(5000) % 63
    v = sv.loop_guard(torch.from_numpy(t).to(DEV))
    np.testing.assert_array_equal(v.cpu().numpy(), O.repeating(t))


def _incremental_verdicts(sv, row, window, repeats, every=16, dtype=torch.int64):
    """Verdicts of the incremental guard at lengths every, 2*every, ... of one row,
    entering the new windows at each check."""
    t = torch.from_numpy(row).to(DEV).to(dtype)
    table = sv.ops.guard_table(len(row), DEV)
    out = torch.zeros(len(row) // every, dtype=torch.uint8, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    prev = 0
    for k, n in enumerate(range(every, len(row) + 1, every)):
        sv.ops.loop_guard_incremental(table, t, prev, n, window, repeats, out=out[k:k + 1], status=status)
        prev = n
    assert int(status) == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("window,repeats", [(1, 3), (8, 2), (64, 3), (64, 5), (200, 3)])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_incremental_matches_batched_at_every_check(sv, window, repeats, dtype):
    """The incremental guard's verdict after each block of 16 tokens equals the
    full rescan (oracle) of the same prefix: tiny alphabets (many hash-equal
    windows), planted repeats, periodic and constant stretches."""
    g = np.random.default_rng(window + repeats)
    rows = [g.integers(0, 3, 1600), g.integers(0, 40000, 1600), np.ones(1600, np.int64),
            np.arange(1600) % 37, np.concatenate([g.integers(0, 9, 700), np.tile(g.integers(0, 9, 80), 12)[:900]])]
    for row in rows:
        row = row.astype(np.int64)
        got = _incremental_verdicts(sv, row, window, repeats, dtype=dtype)
        lengths = np.arange(16, len(row) + 1, 16, dtype=np.int32)
        want = O.repeating(np.broadcast_to(row.astype(np.int32), (len(lengths), len(row))).copy(), lengths, window,
                           repeats)
        np.testing.assert_array_equal(got, want)


def test_incremental_built_at_once_on_cfg5(sv):
    """The whole table entered in one call (insert_from = 0) gives the reference's
    verdicts on config 5's 16384-token rows."""
    t, verdict = cfg5_fixture()
    out = torch.zeros(len(t), dtype=torch.uint8, device=DEV)
    for r in range(0, len(t), 8):
        table = sv.ops.guard_table(t.shape[1], DEV)
        sv.ops.loop_guard_incremental(table, torch.from_numpy(t[r]).to(DEV), 0, t.shape[1], out=out[r:r + 1])
    np.testing.assert_array_equal(out.cpu().numpy()[::8], verdict[::8])


def test_incremental_reports_a_full_table(sv):
    row = torch.arange(300, dtype=torch.int64, device=DEV)
    table = torch.full((64,), -1, dtype=torch.int64, device=DEV)  # room for 64 of 237 windows
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    sv.ops.loop_guard_incremental(table, row, 0, 300, out=torch.zeros(1, dtype=torch.uint8, device=DEV),
                                  status=status)
    assert int(status) == sv._lib.ST_GUARD_FULL
