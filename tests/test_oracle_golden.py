"""Pin the CPU oracle to the reference: golden vectors made by running the
reference's own functions (tests/golden/make_golden.py).

Bars (north star): kept sets exact except at exact ties / top-p rounding
boundaries; warped scores bit-exact in sample mode (penalty and temperature are
IEEE fp32 operations in both); probabilities within 1e-6 relative.  In beam mode
the reference's log_softmax rounds differently from the oracle's exact
normaliser (a per-beam constant of at most 2^-17, from its fp32 sum over V terms),
so log-probs are compared within that constant plus 4 ulp, and probabilities within
the rounding of the fp32 scores they come from.
"""
import numpy as np
import pytest
import torch

from _golden import cfg5_fixture, explain_mismatch, load, names, row_sparse, tempered
from oracle import oracle as O

PROB_RTOL = 1e-6


@pytest.mark.parametrize("name", names("proc"))
def test_sample_chain_matches_reference(name):
    d = load(name)
    x, seen = d["logits"], d["seen"]
    R, V = x.shape
    T, p, keep = float(d["temperature"]), float(d["top_p"]), int(d["keep"])
    out = O.sample(x, np.full(R, 0.5, np.float32), seen=seen, temperature=T, top_p=p, keep=keep, dense=True)
    assert (out["status"] == 0).all()
    for r in range(R):
        gi, gv = row_sparse(d, r)
        _, gp = row_sparse(d, r, "prob")
        oi = np.nonzero(np.isfinite(out["scores"][r]))[0]
        why = explain_mismatch(tempered(x[r], seen[r], T), oi, gi, p, keep)
        assert why is None, f"{name} row {r}: {why}"
        common = np.intersect1d(oi, gi)
        sel = np.isin(gi, common)
        # Warped scores: identical IEEE operations -> bit-exact.
        np.testing.assert_array_equal(out["scores"][r][gi[sel]], gv[sel])
        if len(common) == len(gi) == len(oi):
            np.testing.assert_allclose(out["probs"][r][gi], gp, rtol=PROB_RTOL, atol=1e-30)


@pytest.mark.parametrize("name", names("beam"))
def test_beam_chain_matches_reference(name):
    d = load(name)
    x, seen, running = d["logits"], d["seen"], d["running"]
    B, V = x.shape
    T, p = float(d["temperature"]), float(d["top_p"])
    out = O.beam(x, running, np.full(2 * B, 0.5, np.float32), seen=seen, temperature=T, top_p=p)
    assert out["status"] == 0
    # The log-normaliser: exact fixed-point sum + double log vs torch's fp32 logsumexp.
    np.testing.assert_allclose(out["max"] + out["lognorm"], d["logsumexp"], rtol=4e-7)
    all_same = True
    for b in range(B):
        gi, gv = row_sparse(d, b)
        lp = out["logp"][b]
        oi = np.nonzero(np.isfinite(lp))[0]
        # Recompute the oracle's pre-top-k values to judge boundary cases.
        s = tempered((x[b] - out["max"][b]) - out["lognorm"][b], seen[b], T)
        why = explain_mismatch(s, oi, gi, p, 2)
        assert why is None, f"{name} beam {b}: {why}"
        same = set(oi) == set(gi)
        all_same &= same
        if same:
            # lp = (x - M) - L.  The reference's normaliser L is an fp32 sum of V
            # exponentials, the oracle's an exact one: they differ by a per-beam
            # constant (times the penalty on seen entries, over the temperature),
            # bounded here by 2^-17 in the log-prob.  What remains is the rounding of
            # x - M and of L (scaled by the penalty and temperature) plus the last
            # rounding.
            diff = (lp[gi] - gv).astype(np.float64)
            scale = np.where(seen[b][gi], 3.1, 1.0)
            off = float(np.median(diff / scale))
            assert abs(off) <= 2.0 ** -17, f"{name} beam {b}: normaliser offset {off}"
            xm = np.abs(x[b][gi] - out["max"][b]).astype(np.float32)
            carry = (np.spacing(xm) + np.spacing(np.float32(abs(out["lognorm"][b])))) * 3.1 / T
            tol = 4 * (np.spacing(np.abs(gv).astype(np.float32)) + carry)
            assert np.all(np.abs(diff - off * scale) <= tol), f"{name} beam {b} log-probs"
    if all_same:
        assert out["nnz"] == int(d["nnz"])
        probs = out["probs"]
        nz = d["prob_idx"]
        np.testing.assert_array_equal(np.nonzero(probs)[0], nz)
        scores = np.concatenate([out["logp"][b] + np.float32(running[b]) for b in range(B)])[nz]
        # fp32 scores (log-prob + running score) carry |score| * 2^-24 of rounding.
        rtol = np.maximum(PROB_RTOL, 8 * np.abs(scores) * 2.0 ** -24)
        assert np.all(np.abs(probs[nz] - d["prob_val"]) <= rtol * d["prob_val"] + 1e-37), name


def test_loop_guard_matches_reference():
    d = np.load(load.__globals__["GOLDEN"] + "/repeat.npz")
    v = O.repeating(d["tokens"], d["lengths"])
    np.testing.assert_array_equal(v, d["verdict"])


def test_loop_guard_matches_reference_cfg5():
    """Config 5 at full size: 256 rows of 16384 tokens (planted and random halves)."""
    t, verdict = cfg5_fixture()
    np.testing.assert_array_equal(O.repeating(t), verdict)
    assert verdict[:128].all() and not verdict[128:].any()


def test_exp_accuracy():
    x = np.concatenate([np.linspace(-87.3, 0, 400001), np.linspace(0, 88.7, 1001)]).astype(np.float32)
    y = O.exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    err = np.abs(y - ref) / np.spacing(ref.astype(np.float32))
    assert err.max() < 1.0
    assert O.exp(np.array([0.0, -np.inf, np.nan], np.float32))[:2].tolist() == [1.0, 0.0]
    assert np.isnan(O.exp(np.array([np.nan], np.float32))[0])
    # Never above 1 for x <= 0, and non-increasing towards -inf.
    xs = -np.sort(np.random.default_rng(0).exponential(10, 100000).astype(np.float32))
    ys = O.exp(xs)
    assert ys.max() <= 1.0 and np.all(np.diff(ys) <= 0)


def test_log_fixed_is_correctly_rounded():
    rng = np.random.default_rng(1)
    s = np.concatenate([rng.integers(2 ** 44, 2 ** 62, 20000, dtype=np.uint64),
                        np.array([2 ** 44, 2 ** 45, 3 * 2 ** 44], np.uint64)])
    got = O.log_fixed(s).astype(np.float64)
    ref = np.log(s.astype(np.float64) / 2 ** 44)
    assert np.all(np.abs(got - ref) <= 0.5 * np.spacing(np.abs(ref).astype(np.float32)) + 1e-300)


def test_mulfloor_exact():
    from fractions import Fraction
    rng = np.random.default_rng(2)
    a = rng.integers(0, 2 ** 63, 2000, dtype=np.uint64)
    f = rng.random(2000).astype(np.float32)
    f[:5] = [0.0, 1e-45, 0.1, np.nextafter(np.float32(1), np.float32(0)), 0.5]
    got = O.mulfloor(a, f)
    for i in range(len(a)):
        assert int(got[i]) == int(Fraction(int(a[i])) * Fraction(float(f[i])))


def test_draw_distribution_matches_torch_multinomial():
    """The supplied-uniform inverse-CDF draw and torch.multinomial (the reference's
    draw, runtime_shared.py:201) sample the same distribution (chi-square)."""
    d = load("proc_grid0")
    x, seen = d["logits"][:1], d["seen"][:1]
    n = 20000
    u = np.random.default_rng(3).random(n).astype(np.float32)
    out = O.sample(np.repeat(x, n, 0), u, seen=np.repeat(seen, n, 0), temperature=0.7, top_p=0.9, cap=0)
    ours = np.bincount(out["token"], minlength=x.shape[1])
    gi, _ = row_sparse(d, 0)
    _, gp = row_sparse(d, 0, "prob")
    probs = torch.zeros(x.shape[1])
    probs[torch.from_numpy(gi.astype(np.int64))] = torch.from_numpy(gp)
    g = torch.Generator().manual_seed(4)
    theirs = np.bincount(torch.multinomial(probs.expand(n, -1), 1, generator=g)[:, 0].numpy(), minlength=x.shape[1])
    k = gi
    expect = gp.astype(np.float64) * n
    ok = expect >= 5
    for counts in (ours, theirs):
        chi2 = (((counts[k][ok] - expect[ok]) ** 2) / expect[ok]).sum()
        dof = ok.sum() - 1
        assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)
    assert set(np.nonzero(ours)[0]) <= set(gi)
