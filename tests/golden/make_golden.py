"""Generate golden vectors by running the reference's own sampling functions.

    python tests/golden/make_golden.py --reference /path/to/ComfyUI-StarVector-GGUF [--only big]
    (or with STARVECTOR_REF=/path/to/ComfyUI-StarVector-GGUF in the environment)

Imports the unmodified reference (ComfyUI-StarVector-GGUF, runtime_shared.py) as
the package `starvector_node`, the way its own tests do (tests/package_alias.py),
runs its CPU torch implementation on seeded inputs and writes compressed .npz
fixtures next to this script.  Needs the reference checkout, torch and
transformers; the fixtures it writes are what the tests read (the reference does
not exist on the GPU box).

Fixtures:
  proc_<case>.npz  _warp(_penalize(x, seen), T, top_p, keep)  (runtime_shared.py:170-187)
                   and its softmax, stored sparse (kept indices / values / probs).
  beam_<case>.npz  the beam step of runtime_shared.py:230-235: log_probs, the
                   softmax over beams*V and count_nonzero, stored sparse.
  repeat.npz       _repeating verdicts (runtime_shared.py:156-167).
The full-size BASELINE configurations (a 16-row slice of config 4 with Zipf
histories, config 3's eight bf16 beams at V=49152, config 5's 256 loop-guard rows
of 16384 tokens) are too large to store: their fixtures (proc_cfg4z, beam_cfg3,
repeat_cfg5) hold the reference's outputs plus the generator (bench.py's seeded
workload functions), its arguments and a SHA-256 of the generated inputs, which
the tests regenerate and check.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
V_BIG = 49152


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference(path):
    pkg = types.ModuleType("starvector_node")
    pkg.__path__ = [path]
    sys.modules["starvector_node"] = pkg
    from starvector_node import runtime_shared
    return runtime_shared


def history_ids(rng, n, vocab, repeat_frac=0.3):
    """n ids: (1 - repeat_frac) uniform in [0, vocab), the rest copies of earlier ids."""
    ids = rng.integers(0, vocab, n)
    for j in range(1, n):
        if rng.random() < repeat_frac:
            ids[j] = ids[rng.integers(0, j)]
    return ids.astype(np.int32)


def seen_of(ids_rows, vocab):
    seen = np.zeros((len(ids_rows), vocab), bool)
    for r, ids in enumerate(ids_rows):
        seen[r, ids] = True
    return seen


def sparse_rows(dense, keep_mask):
    """Concatenate per-row kept entries: (offsets [R+1], idx, values)."""
    offs, idx, vals = [0], [], []
    for r in range(dense.shape[0]):
        k = np.nonzero(keep_mask[r])[0]
        idx.append(k.astype(np.int32))
        vals.append(dense[r, k].astype(np.float32))
        offs.append(offs[-1] + len(k))
    return np.array(offs, np.int64), np.concatenate(idx), np.concatenate(vals)


def proc_case(rs, name, logits, seen, temperature, top_p, keep, extra=None, store_inputs=True):
    x = torch.from_numpy(logits.astype(np.float32))
    s = torch.from_numpy(seen)
    warped = rs._warp(rs._penalize(x, s), temperature, top_p, keep)
    probs = warped.softmax(-1)
    w = warped.numpy()
    p = probs.numpy()
    kept = np.isfinite(w)
    offs, idx, vals = sparse_rows(w, kept)
    _, _, pv = sparse_rows(p, kept)
    out = dict(vocab=np.int64(seen.shape[1]), temperature=np.float64(temperature), top_p=np.float64(top_p),
               keep=np.int64(keep), offs=offs, idx=idx, val=vals, prob=pv)
    if store_inputs:
        out.update(logits=logits.astype(np.float32), seen=np.packbits(seen, axis=1))
    if extra:
        out.update(extra)
    np.savez_compressed(os.path.join(HERE, f"proc_{name}.npz"), **out)
    print(f"proc_{name}: rows={logits.shape[0]} V={logits.shape[1]} kept={np.diff(offs).tolist()[:8]}")


def beam_case(rs, name, logits, seen, running, temperature=1.5, top_p=0.9, extra=None):
    x = torch.from_numpy(logits.astype(np.float32))
    s = torch.from_numpy(seen)
    B, V = x.shape
    # runtime_shared.py:230-235, the device part of one beam step.
    log_probs = rs._warp(rs._penalize(torch.log_softmax(x, -1), s), temperature, top_p, 2)
    scores = (log_probs + torch.tensor(list(map(float, running)))[:, None]).view(1, -1)
    probs = scores.softmax(-1)
    nnz = int(torch.count_nonzero(probs))
    lp = log_probs.numpy()
    kept = np.isfinite(lp)
    offs, idx, vals = sparse_rows(lp, kept)
    pf = probs.numpy()[0]
    nz = np.nonzero(pf)[0]
    out = dict(vocab=np.int64(V), running=np.asarray(running, np.float64), temperature=np.float64(temperature),
               top_p=np.float64(top_p), offs=offs, idx=idx, val=vals, prob_idx=nz.astype(np.int64),
               prob_val=pf[nz].astype(np.float32), nnz=np.int64(nnz),
               logsumexp=torch.logsumexp(x, -1).numpy().astype(np.float32))
    if extra is None:
        out.update(logits=logits.astype(np.float32), seen=np.packbits(seen, axis=1))
    else:
        out.update(extra)
    np.savez_compressed(os.path.join(HERE, f"beam_{name}.npz"), **out)
    print(f"beam_{name}: B={B} V={V} kept={np.diff(offs).tolist()} nnz={nnz}")


def big_cases(rs):
    """The full-size configurations, inputs regenerated from bench.py's generators."""
    sys.path.insert(0, ROOT)
    import bench
    # A 16-row slice of config 4: Zipf(1.1) histories of 4096 ids, T 1.5, top-p 0.9.
    d = bench.cfg4(seed=11, rows=16)
    seen = seen_of(d["history"], V_BIG)
    proc_case(rs, "cfg4z", d["logits"], seen, 1.5, 0.9, 1, store_inputs=False,
              extra=dict(gen="cfg4", gen_seed=np.int64(11), gen_rows=np.int64(16),
                         sha=digest(d["logits"], d["history"])))
    # Config 3: 8 beams, bf16-valued N(0,3^2) logits with 1 % of ids +6, V=49152,
    # histories of 8000 ids, running scores U(-200,-10).
    d = bench.cfg3(seed=12)
    beam_case(rs, "cfg3", d["logits"], seen_of(d["history"], V_BIG), d["running"],
              extra=dict(gen="cfg3", gen_seed=np.int64(12), sha=digest(d["logits"], d["history"])))
    print("beam_cfg3 written")
    # Config 5: 256 rows of 16384 tokens, the first half ending in a window repeated 3 times.
    t = bench.cfg5_tokens(seed=13)
    verdict = np.array([rs._repeating(row.tolist()) for row in t], bool)
    np.savez_compressed(os.path.join(HERE, "repeat_cfg5.npz"), verdict=verdict, gen="cfg5_tokens",
                        gen_seed=np.int64(13), sha=digest(t))
    print("repeat_cfg5:", int(verdict.sum()), "of", len(verdict), "repeating")


def main(path, only=None):
    rs = load_reference(path)
    if only == "big":
        big_cases(rs)
        return
    rng = np.random.default_rng(20261201)

    # The reference's own processor pin (tests/test_generation.py:109-122).
    torch.manual_seed(0)
    scores = (torch.randn(3, 200) * 4).numpy()
    history = np.array([[5, 9, 9], [0, 1, 2], [7, 150, 199]])
    seen = seen_of(history, 200)
    for keep in (1, 2):
        proc_case(rs, f"hfpin_keep{keep}", scores, seen, 1.5, 0.9, keep)

    # B=1, V=49152, 2*N(0,1) with 20 ids boosted by +8, history of
    # 1024 ids with 30 % repeats; rep 3.1, T 1.5, top-k 50, top-p 0.9.
    x = (2.0 * rng.standard_normal((1, V_BIG))).astype(np.float32)
    x[0, rng.choice(V_BIG, 20, replace=False)] += 8.0
    h = history_ids(rng, 1024, V_BIG)
    proc_case(rs, "cfg1", x, seen_of([h], V_BIG), 1.5, 0.9, 1, extra=dict(history=h))

    # A grid of temperatures / top_p / keep on V=1000 rows.
    combos = [(0.7, 0.9, 1), (1.0, 0.9, 1), (1.5, 0.5, 2), (2.5, 0.97, 1), (1.5, 1.0, 1), (1.5, 0.9, 2),
              (0.3, 0.99, 1), (4.0, 0.6, 2)]
    for c, (t, p, k) in enumerate(combos):
        x = (rng.standard_normal((8, 1000)) * rng.uniform(0.5, 4.0, (8, 1))).astype(np.float32)
        hs = [rng.integers(0, 1000, rng.integers(0, 300)) for _ in range(8)]
        proc_case(rs, f"grid{c}", x, seen_of(hs, 1000), t, p, k)

    # fp16-valued logits: many exact ties around the 50th value.
    x = (rng.standard_normal((8, 5000)) * 3).astype(np.float16).astype(np.float32)
    x = np.round(x * 4) / 4
    hs = [rng.integers(0, 5000, 400) for _ in range(8)]
    proc_case(rs, "ties", x.astype(np.float32), seen_of(hs, 5000), 1.5, 0.9, 1)

    # ScriptDecoder-like rows (tests/test_generation.py:21-49): zeros and one 200.
    x = np.zeros((3, 128), np.float32)
    x[0, 7] = 200.0
    x[1, 3] = 200.0
    x[2, 100] = 200.0
    proc_case(rs, "script", x, seen_of([[7, 8], [], [1, 2, 100]], 128), 1.5, 0.9, 1)

    # Rows with many -inf logits (fewer finite entries than top_k).
    x = rng.standard_normal((4, 300)).astype(np.float32) * 2
    for r in range(4):
        x[r, rng.choice(300, 300 - [10, 49, 51, 200][r], replace=False)] = -np.inf
    proc_case(rs, "neginf", x, seen_of([rng.integers(0, 300, 30) for _ in range(4)], 300), 1.5, 0.9, 1)

    # Beam steps.  2 beams, V=49152, N(0,2^2), histories 2048,
    # running scores U(-200,-10).
    x = (2.0 * rng.standard_normal((2, V_BIG))).astype(np.float32)
    hs = [rng.integers(0, V_BIG, 2048) for _ in range(2)]
    beam_case(rs, "cfg2", x, seen_of(hs, V_BIG), rng.uniform(-200, -10, 2))
    # First step of _beam_sample: running scores [0, -1e9] (runtime_shared.py:225) and
    # the prefill's stride-0 expanded logits (runtime_1b.py:82): identical rows.
    beam_case(rs, "first", np.repeat(x[:1, :8192], 2, axis=0), seen_of([[], []], 8192), [0.0, -1e9])
    # 8 beams, bf16-valued N(0,3^2) with a heavy tail (1 % of ids +6), V=4096.
    x = (3.0 * rng.standard_normal((8, 4096))).astype(np.float32)
    x[:, rng.choice(4096, 41, replace=False)] += 6.0
    x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    hs = [rng.integers(0, 4096, 800) for _ in range(8)]
    beam_case(rs, "b8", x, seen_of(hs, 4096), rng.uniform(-30, -10, 8))
    # Beams whose running scores differ by more than the fp32 exp range.
    x = (2.0 * rng.standard_normal((4, 1000))).astype(np.float32)
    beam_case(rs, "spread", x, seen_of([rng.integers(0, 1000, 50) for _ in range(4)], 1000),
              [-10.0, -95.0, -120.0, -1e9])
    # ScriptDecoder-like beams: huge ties.
    x = np.zeros((2, 128), np.float32)
    x[:, 7] = 200.0
    beam_case(rs, "script", x, seen_of([[7], [3]], 128), [0.0, -1e9])

    # Loop guard verdicts.
    rows = []
    script = list(range(5, 69)) * 20
    for L in (0, 63, 64, 191, 192, 193, 200, 255, 256, 300, 1000):
        rows.append(script[:L])
    for L in (192, 500, 2560, 5000):
        rows.append(rng.integers(0, 49152, L).tolist())
    for L, reps in ((1000, 3), (1000, 2), (3000, 3), (3000, 4)):
        t = rng.integers(0, 49152, L)
        win = rng.integers(0, 49152, 64)
        pos = sorted(rng.choice(np.arange(0, L - 64 - 64, 97), reps - 1, replace=False).tolist())
        for p in pos:
            t[p:p + 64] = win
        t[L - 64:] = win
        rows.append(t.tolist())
    t = [1] * 400
    rows.append(t)
    t = ([1] * 63 + [2]) * 5
    rows.append(t)
    lengths = np.array([len(r) for r in rows], np.int32)
    mat = np.zeros((len(rows), max(lengths)), np.int32)
    for i, r in enumerate(rows):
        mat[i, :len(r)] = r
    verdict = np.array([rs._repeating(list(r)) for r in rows], bool)
    np.savez_compressed(os.path.join(HERE, "repeat.npz"), tokens=mat, lengths=lengths, verdict=verdict)
    print("repeat:", verdict.astype(int).tolist())
    big_cases(rs)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("STARVECTOR_REF"),
                    help="checkout of ComfyUI-StarVector-GGUF (or STARVECTOR_REF)")
    ap.add_argument("--only", choices=["big"], default=None, help="write only the full-size fixtures")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set STARVECTOR_REF")
    main(args.reference, args.only)
