"""The CPU baseline's torch chain (oracle/torch_chain.py) against the reference-run
golden vectors: bench.py times the reference's own computation."""
import numpy as np
import pytest
import torch

from _golden import load, names, row_sparse
from oracle import torch_chain as TC


@pytest.mark.parametrize("name", names("proc"))
def test_warp_matches_reference_goldens(name):
    d = load(name)
    x = torch.from_numpy(d["logits"].astype(np.float32))
    seen = torch.from_numpy(d["seen"])
    out = TC.warp(TC.penalize(x, seen), float(d["temperature"]), float(d["top_p"]), int(d["keep"]))
    probs = out.softmax(-1).numpy()
    out = out.numpy()
    for r in range(out.shape[0]):
        idx, val = row_sparse(d, r)
        _, prob = row_sparse(d, r, "prob")
        kept = np.nonzero(np.isfinite(out[r]))[0]
        np.testing.assert_array_equal(kept, idx)
        np.testing.assert_array_equal(out[r, kept], val)
        np.testing.assert_allclose(probs[r, kept], prob, rtol=1e-6)


def test_sample_step_keeps_the_draw_inside_the_kept_set():
    g = np.random.default_rng(0)
    x = torch.from_numpy((2 * g.standard_normal((4, 3000))).astype(np.float32))
    seen = TC.seen_mask(g.integers(0, 3000, (4, 200)), 3000)
    kept = np.isfinite(TC.warp(TC.penalize(x, seen), 1.5, 0.9, 1).numpy())
    before = seen.clone()
    tok = TC.sample_step(x, seen, generator=torch.Generator().manual_seed(1)).numpy()
    for r in range(4):
        assert kept[r, tok[r]]
        assert seen[r, tok[r]] and (seen[r].sum() - before[r].sum()) <= 1
