"""Helpers shared by the parity tests: golden fixtures and kept-set comparison.

Kept sets are compared exactly, except where the reference's own result depends on
rounding or on tie order, which the north-star parity bar exempts:
  * top-p boundary: the reference accumulates the top-p mass with an fp32 cumsum
    (runtime_shared.py:184), the oracle exactly; a cut within `margin` of the
    threshold may fall one element either way;
  * exact ties: torch's CPU sort is unstable, so which members of a tie group at
    the top-p cut are removed is unspecified in the reference.
"""
from __future__ import annotations

import glob
import hashlib
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOP_K = 50
REP = 3.1


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {k: z[k] for k in z.files}
    V = int(d["vocab"])
    if "gen" in d:
        d.update(regenerate(d))
    else:
        d["seen"] = np.unpackbits(d["seen"], axis=1)[:, :V].astype(bool)
    return d


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def regenerate(d):
    """Inputs of a full-size fixture from bench.py's seeded generators, checked
    against the digest the generator script stored (tests/golden/make_golden.py)."""
    import bench
    gen, seed = str(d["gen"]), int(d["gen_seed"])
    if gen == "cfg4":
        w = bench.cfg4(seed=seed, rows=int(d["gen_rows"]))
    elif gen == "cfg3":
        w = bench.cfg3(seed=seed)
    else:
        raise ValueError(gen)
    assert digest(w["logits"], w["history"]) == str(d["sha"]), f"{gen}: generator output changed"
    V = int(d["vocab"])
    seen = np.zeros((w["logits"].shape[0], V), bool)
    for r, ids in enumerate(w["history"]):
        seen[r, ids] = True
    return dict(logits=w["logits"], seen=seen, history=w["history"])


def cfg5_fixture():
    """Config 5's tokens (regenerated, digest-checked) and the reference's verdicts."""
    import bench
    z = np.load(os.path.join(GOLDEN, "repeat_cfg5.npz"))
    t = bench.cfg5_tokens(seed=int(z["gen_seed"]))
    assert digest(t) == str(z["sha"]), "cfg5_tokens output changed"
    return t, z["verdict"]


def names(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "_*.npz")))


def row_sparse(d, r, key="val"):
    a, b = int(d["offs"][r]), int(d["offs"][r + 1])
    out = d["idx"][a:b], d[key][a:b]
    return out


def tempered(x, seen, temperature, rep=REP):
    """pen(x)/T in fp32 exactly as runtime_shared.py:170-179 computes it."""
    x = x.astype(np.float32)
    T = np.float32(temperature)
    r = np.float32(rep)
    pen = np.where(x < 0, x * r, x / r).astype(np.float32)
    s = np.where(seen, pen, x).astype(np.float32)
    return (s / T).astype(np.float32)


def explain_mismatch(s, kept_a, kept_b, top_p, keep, margin=2e-5, top_k=TOP_K):
    """None if kept sets a and b (index arrays) differ only at an exact tie or at a
    top-p cut within `margin` of the threshold; else a description of the failure."""
    a, b = set(map(int, kept_a)), set(map(int, kept_b))
    if a == b:
        return None
    diff = sorted(a ^ b)
    kk = max(top_k, keep)
    thr = np.sort(s)[::-1][kk - 1]
    surv = np.nonzero(s >= thr)[0]
    order = surv[np.lexsort((surv, s[surv]))]
    vals = s[order]
    pos = {int(i): j for j, i in enumerate(order)}
    if any(d not in pos for d in diff):
        return f"difference outside the top-k survivors: {diff[:8]}"
    dvals = {float(s[d]) for d in diff}
    if len(dvals) == 1 and np.count_nonzero(vals == dvals.pop()) > 1 and len(a) == len(b):
        return None
    M = vals.max()
    w = np.exp(vals.astype(np.float64) - M)
    cum = np.cumsum(w) / w.sum()
    pthr = float(np.float32(1.0 - top_p))
    lo = min(pos[d] for d in diff)
    hi = max(pos[d] for d in diff)
    near = np.abs(cum[max(lo - 1, 0):hi + 1] - pthr)
    if near.min() <= margin:
        return None
    return f"kept sets differ at sorted positions {lo}..{hi}, cumulative mass margin {near.min():.3g}"
