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
