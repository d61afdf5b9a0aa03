"""GPU parity of the beam step (runtime_shared.py:230-237) against the oracle,
through the C ABI (ops.beam_step -> sv_beam_step): picks, picked scores, pick
count, per-beam kept sets, warped log-probs and probabilities, bit for bit."""
import numpy as np
import pytest
import torch

import bench
from _golden import explain_mismatch, load, names, row_sparse, tempered
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def run_both(sv, x, running, u, seen=None, ids=None, dtype=torch.float32, T=1.5, p=0.9, top_k=50, keep=2,
             npick=None, force=False, cap=256):
    B, Vv = x.shape
    xd = to_dev(x).to(dtype)
    xf = xd.float().cpu().numpy()
    kw = {}
    if ids is not None:
        kw["history"] = to_dev(ids.astype(np.int32))
        seen = O.seen_from_ids(ids, np.full(B, ids.shape[1]), Vv)
    elif seen is not None:
        kw["seen"] = to_dev(seen.astype(bool))
    npick = 2 * B if npick is None else npick
    out = sv.beam_step(xd, to_dev(np.asarray(running, np.float32)), to_dev(u), temperature=T, top_p=p, top_k=top_k,
                       keep=keep, num_picks=npick, out_capacity=cap, dense_logprob=True, force_general=force, **kw)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in out.items()}
    ref = O.beam(xf, running, u, seen=seen, temperature=T, top_p=p, top_k=top_k, keep=keep, npick=npick)
    return got, ref


def assert_same(got, ref):
    assert int(got["status"][0]) == ref["status"]
    if ref["status"]:
        assert int(got["n"][0]) == 0
        return
    n = int(got["n"][0])
    assert n == ref["n"]
    np.testing.assert_array_equal(got["picks"][:n], ref["picks"])
    np.testing.assert_array_equal(got["scores"][:n], ref["scores"])
    B = got["kept_count"].shape[0]
    cap = got["kept_idx"].shape[1]
    V = ref["logp"].shape[1]
    for b in range(B):
        ki = np.nonzero(np.isfinite(ref["logp"][b]))[0]
        assert got["kept_count"][b] == len(ki)
        k = min(len(ki), cap)
        np.testing.assert_array_equal(got["kept_idx"][b, :k], ki[:k])
        np.testing.assert_array_equal(got["kept_logprob"][b, :k], ref["logp"][b][ki[:k]])
        np.testing.assert_array_equal(got["kept_prob"][b, :k], ref["probs"][b * V + ki[:k]])
    np.testing.assert_array_equal(got["dense_logprob"], ref["logp"])


@pytest.mark.parametrize("force", [False, True], ids=["fast", "general"])
@pytest.mark.parametrize("name", names("beam"))
def test_golden_beam_cases(sv, name, force):
    d = load(name)
    x, seen, running = d["logits"], d["seen"], d["running"].astype(np.float32)
    B = x.shape[0]
    u = np.random.default_rng(3).random(2 * B).astype(np.float32)
    got, ref = run_both(sv, x, running, u, seen=seen, T=float(d["temperature"]), p=float(d["top_p"]), force=force)
    assert_same(got, ref)
    lp = got["dense_logprob"]
    for b in range(B):
        gi, _ = row_sparse(d, b)
        oi = np.nonzero(np.isfinite(lp[b]))[0]
        s = tempered((x[b] - ref["max"][b]) - ref["lognorm"][b], seen[b], float(d["temperature"]))
        assert explain_mismatch(s, oi, gi, float(d["top_p"]), 2) is None


def test_cfg2_two_beams(sv):
    d = bench.cfg2()
    got, ref = run_both(sv, d["logits"], d["running"], d["uniforms"], ids=d["history"])
    assert_same(got, ref)


@pytest.mark.parametrize("force", [False, True], ids=["fast", "general"])
def test_cfg3_eight_beams_bf16(sv, force):
    d = bench.cfg3()
    got, ref = run_both(sv, d["logits"], d["running"], d["uniforms"], ids=d["history"], dtype=torch.bfloat16,
                        force=force)
    assert_same(got, ref)


@pytest.mark.parametrize("beams", [1, 3, 8, 16])
def test_beam_counts_and_first_step(sv, beams):
    g = np.random.default_rng(beams)
    Vv = 6000
    row = (2 * g.standard_normal((1, Vv))).astype(np.float32)
    x = np.repeat(row, beams, 0)
    running = np.array([0.0] + [-1e9] * (beams - 1), np.float32)
    u = g.random(2 * beams).astype(np.float32)
    got, ref = run_both(sv, x, running, u, dtype=torch.float16)
    assert_same(got, ref)
    # Stride-0 logits (the prefill's expand) give the same result.
    xd = to_dev(row).half().expand(beams, -1)
    out = sv.beam_step(xd, to_dev(running), to_dev(u))
    n = int(out["n"].item())
    np.testing.assert_array_equal(out["picks"][:n].cpu().numpy(), ref["picks"])


def test_fewer_possible_continuations_than_picks(sv):
    """count_nonzero(probs) < 2*beams (runtime_shared.py:233-235): a dominant token
    and beams far behind."""
    x = np.zeros((4, 500), np.float32)
    x[:, 3] = 200.0
    running = np.array([0.0, -1e9, -1e9, -1e9], np.float32)
    u = np.full(8, 0.3, np.float32)
    got, ref = run_both(sv, x, running, u)
    assert ref["n"] < 8
    assert_same(got, ref)


def test_spread_running_scores_and_npick(sv):
    g = np.random.default_rng(4)
    x = (2 * g.standard_normal((5, 3000))).astype(np.float32)
    running = np.array([-10, -95, -120, -60, -1e9], np.float32)
    for npick in (1, 5, 10):
        u = g.random(npick).astype(np.float32)
        got, ref = run_both(sv, x, running, u, ids=g.integers(0, 3000, (5, 100)), npick=npick)
        assert_same(got, ref)


def test_beam_errors(sv):
    x = np.zeros((2, 300), np.float32)
    x[1, 4] = np.nan
    got, ref = run_both(sv, x, np.zeros(2, np.float32), np.full(4, 0.5, np.float32))
    assert int(got["status"][0]) == 1 and ref["status"] == 1
    x = np.full((2, 300), -np.inf, np.float32)
    got, ref = run_both(sv, x, np.zeros(2, np.float32), np.full(4, 0.5, np.float32))
    assert int(got["status"][0]) == 3 and ref["status"] == 3


def test_workspace_reuse_across_calls(sv):
    """The merge counter resets itself: repeated calls on one workspace agree."""
    d = bench.cfg2()
    x, rs, u, h = (to_dev(d[k]) for k in ("logits", "running", "uniforms", "history"))
    first = sv.beam_step(x, rs, u, history=h)
    picks = first["picks"].clone()
    for _ in range(5):
        o = sv.beam_step(x, rs, u, history=h)
        assert torch.equal(o["picks"], picks)


@pytest.mark.parametrize("force", [False, True], ids=["warp", "block"])
@pytest.mark.parametrize("beams,top_k", [(1, 50), (2, 50), (2, 64), (3, 30), (8, 12), (16, 6), (32, 3)])
def test_register_merge_shapes(sv, beams, top_k, force):
    """Kept lists that fit the one-warp register merge (lanes split across beams)
    and the same inputs through the block merge; several seeds each."""
    for seed in range(3):
        g = np.random.default_rng(100 + 7 * beams + seed)
        x = (2 * g.standard_normal((beams, 2048))).astype(np.float32)
        running = np.sort(g.uniform(-30, 0, beams)).astype(np.float32)[::-1].copy()
        u = g.random(2 * beams).astype(np.float32)
        got, ref = run_both(sv, x, running, u, ids=g.integers(0, 2048, (beams, 300)), top_k=top_k, p=0.97,
                            force=force)
        assert_same(got, ref)


@pytest.mark.parametrize("force", [False, True], ids=["warp", "block"])
@pytest.mark.parametrize("lag", [20.0, 45.0, 70.0])
def test_merge_mass_below_fixed_point(sv, lag, force):
    """One dominant continuation and a second beam far behind: after the first
    pick the remaining candidates have probabilities above zero but no
    fixed-point weight, so the later picks take the largest remaining
    probability (runtime_shared.py:233-235)."""
    g = np.random.default_rng(int(lag))
    x = (2 * g.standard_normal((2, 4096))).astype(np.float32)
    x[0, 17] += 40.0
    running = np.array([0.0, -lag], np.float32)
    u = g.random(4).astype(np.float32)
    got, ref = run_both(sv, x, running, u, force=force)
    assert ref["n"] >= 2
    assert_same(got, ref)


@pytest.mark.parametrize("force", [False, True], ids=["warp", "block"])
@pytest.mark.parametrize("running,vocab,top_p,status", [
    ([np.nan, 0.0], 300, 0.9, 1),      # NaN running score
    ([np.inf, 0.0], 300, 0.9, 1),      # +inf + the -inf outside the kept list
    ([-np.inf, -np.inf], 300, 0.9, 3),  # every score -inf
    ([np.inf, 0.0], 50, 1.0, 2),       # every entry kept: a +inf score
    ([-np.inf, 0.0], 300, 0.9, 0),     # one beam out of the draw
])
def test_nonfinite_running_scores(sv, running, vocab, top_p, status, force):
    """Non-finite running scores give the statuses of the flattened softmax over
    scores = log_probs + running (runtime_shared.py:231-233)."""
    g = np.random.default_rng(vocab)
    x = (2 * g.standard_normal((2, vocab))).astype(np.float32)
    got, ref = run_both(sv, x, np.asarray(running, np.float32), g.random(4).astype(np.float32), p=top_p,
                        force=force)
    assert ref["status"] == status
    assert_same(got, ref)


@pytest.mark.parametrize("force", [False, True], ids=["regs", "block"])
@pytest.mark.parametrize("beams,lag", [(8, 20.0), (8, 45.0), (5, 70.0), (16, 45.0)])
def test_block_register_merge_mass_below_fixed_point(sv, beams, lag, force):
    """Kept lists too long for the one-warp merge but within the block's register
    slots, with beams far behind: draws past the fixed-point mass take the largest
    remaining probability (runtime_shared.py:233-235)."""
    g = np.random.default_rng(beams * 100 + int(lag))
    x = (2 * g.standard_normal((beams, 4096))).astype(np.float32)
    x[0, 17] += 40.0
    running = np.array([0.0] + [-lag] * (beams - 1), np.float32)
    u = g.random(2 * beams).astype(np.float32)
    got, ref = run_both(sv, x, running, u, force=force)
    counts = [int(np.isfinite(ref["logp"][b]).sum()) for b in range(beams)]
    assert max(counts) > 4 * (32 // beams)  # past the one-warp merge
    assert_same(got, ref)
