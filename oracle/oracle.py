"""ctypes bindings of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module,
as the checker.  The functions take numpy arrays and mirror the reference's
sampling chain (ComfyUI-StarVector-GGUF runtime_shared.py:156-265); see
sv_oracle.c for the arithmetic they follow.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .build import LIB, build

OK, ERR_NAN, ERR_POSINF, ERR_ALLNEGINF, ERR_HISTORY, ERR_ARGS = range(6)

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = C.CDLL(LIB)
        P, I64, I32, D, F = C.c_void_p, C.c_int64, C.c_int, C.c_double, C.c_float
        _lib.orc_sample.argtypes = [P, I64, I64, I64, P, P, P, I64, D, D, I32, I32, D, P,
                                    P, P, P, P, I32, P, P, P, I32]
        _lib.orc_sample.restype = I32
        _lib.orc_beam.argtypes = [P, I64, I64, I64, P, P, D, D, I32, I32, D, I32, P,
                                  P, P, P, P, P, P, P, P]
        _lib.orc_beam.restype = I32
        _lib.orc_repeating.argtypes = [P, I64, I64, P, I32, I32, P, I32]
        _lib.orc_repeating.restype = I32
        _lib.orc_exp_vec.argtypes = [P, P, I64]
        _lib.orc_log_fixed_vec.argtypes = [P, P, I64]
        _lib.orc_mulfloor_vec.argtypes = [P, P, P, I64]
        _lib.orc_exp.argtypes = [F]
        _lib.orc_exp.restype = F
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def exp(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_exp_vec(_p(x), _p(y), x.size)
    return y


def log_fixed(s):
    s = np.ascontiguousarray(s, np.uint64)
    y = np.empty(s.shape, np.float32)
    lib().orc_log_fixed_vec(_p(s), _p(y), s.size)
    return y


def mulfloor(a, f):
    a = np.ascontiguousarray(a, np.uint64)
    f = np.ascontiguousarray(np.broadcast_to(np.asarray(f, np.float32), a.shape))
    y = np.empty(a.shape, np.uint64)
    lib().orc_mulfloor_vec(_p(a), _p(f), _p(y), a.size)
    return y


def seen_from_ids(ids, lengths, vocab):
    """Bool [R, V] mask of the ids in each row's history prefix."""
    ids = np.asarray(ids)
    seen = np.zeros((ids.shape[0], vocab), np.uint8)
    for r in range(ids.shape[0]):
        seen[r, ids[r, :lengths[r]]] = 1
    return seen


def sample(logits, uniforms, *, seen=None, ids=None, lengths=None, temperature=1.5, top_p=0.9,
           top_k=50, keep=1, rep_penalty=3.1, cap=None, dense=False, threads=0):
    """Sample-mode step over rows of fp32 logits [R, V].

    History: `seen` bool [R, V] or int32 `ids` [R, H] with `lengths` [R].
    Returns a dict with token [R], count [R], idx/prob [R, cap] (kept tokens in
    ascending index order), status [R], and with dense=True the warped scores
    (the reference's _warp output) and probabilities [R, V].
    """
    x = np.ascontiguousarray(logits, np.float32)
    R, V = x.shape
    u = np.ascontiguousarray(uniforms, np.float32).reshape(R)
    if cap is None:
        cap = V
    token = np.empty(R, np.int64)
    count = np.empty(R, np.int32)
    status = np.empty(R, np.int32)
    oidx = np.full((R, cap), -1, np.int32) if cap else None
    oprob = np.zeros((R, cap), np.float32) if cap else None
    dscores = np.empty((R, V), np.float32) if dense else None
    dprobs = np.empty((R, V), np.float32) if dense else None
    sn = None if seen is None else np.ascontiguousarray(seen, np.uint8)
    idp = lp = None
    hs = 0
    if ids is not None:
        idp = np.ascontiguousarray(ids, np.int32)
        hs = idp.shape[1]
        lp = np.ascontiguousarray(lengths if lengths is not None else np.full(R, hs), np.int32)
    lib().orc_sample(_p(x), R, V, V, _p(sn), _p(idp), _p(lp), hs, float(temperature), float(top_p),
                     int(top_k), int(keep), float(rep_penalty), _p(u), _p(token), _p(count),
                     _p(oidx), _p(oprob), int(cap), _p(dscores), _p(dprobs), _p(status), int(threads))
    out = dict(token=token, count=count, idx=oidx, prob=oprob, status=status)
    if dense:
        out.update(scores=dscores, probs=dprobs)
    return out


def beam(logits, running, uniforms, *, seen=None, temperature=1.5, top_p=0.9, top_k=50, keep=2,
         rep_penalty=3.1, npick=None):
    """One beam-sampling step over logits [B, V] (runtime_shared.py:230-237)."""
    x = np.ascontiguousarray(logits, np.float32)
    B, V = x.shape
    npick = 2 * B if npick is None else npick
    u = np.ascontiguousarray(uniforms, np.float32)
    assert u.size >= npick
    rs = np.ascontiguousarray(running, np.float32).reshape(B)
    sn = None if seen is None else np.ascontiguousarray(seen, np.uint8)
    picks = np.full(npick, -1, np.int64)
    scores = np.zeros(npick, np.float32)
    n = np.zeros(1, np.int32)
    nnz = np.zeros(1, np.int32)
    dlogp = np.empty((B, V), np.float32)
    dprobs = np.empty(B * V, np.float32)
    bmax = np.empty(B, np.float32)
    blog = np.empty(B, np.float32)
    st = lib().orc_beam(_p(x), B, V, V, _p(sn), _p(rs), float(temperature), float(top_p), int(top_k),
                        int(keep), float(rep_penalty), int(npick), _p(u), _p(picks), _p(scores), _p(n),
                        _p(dlogp), _p(dprobs), _p(bmax), _p(blog), _p(nnz))
    k = int(n[0])
    return dict(status=int(st), picks=picks[:k], scores=scores[:k], n=k, nnz=int(nnz[0]),
                logp=dlogp, probs=dprobs, max=bmax, lognorm=blog)


def repeating(tokens, lengths=None, window=64, repeats=3, threads=0):
    """Loop-guard verdicts for rows of int32 tokens [R, L] (runtime_shared.py:156-167)."""
    t = np.ascontiguousarray(tokens, np.int32)
    if t.ndim == 1:
        t = t[None]
    R, L = t.shape
    ln = np.ascontiguousarray(lengths if lengths is not None else np.full(R, L), np.int32)
    v = np.empty(R, np.uint8)
    lib().orc_repeating(_p(t), R, L, _p(ln), int(window), int(repeats), _p(v), int(threads))
    return v.astype(bool)
