"""Tensor-level wrappers of the C ABI (torch CUDA tensors in, torch CUDA tensors out).

Every function enqueues on the current CUDA stream of the tensors' device and does
not synchronise; results are device tensors.  Inputs must be CUDA tensors: there is
no CPU path.  The hot entry points (sample_step, beam_step, beam_advance,
kv_reorder, loop_guard, loop_guard_incremental) go through the thin PyTorch
extension sv_torch (ext/sv_torch.cpp), the others through ctypes (_lib.py); both
call the same C library.
"""
from __future__ import annotations

import torch

from . import _lib as L

_DTYPES = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}


def _need_cuda(t, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the B200 sampling kernels have no CPU path)")


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _rows(logits):
    _need_cuda(logits, "logits")
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    if logits.dtype not in _DTYPES:
        raise ValueError(f"unsupported logits dtype {logits.dtype}")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return logits


def _ptr(t):
    return None if t is None else t.data_ptr()


_EXT = []


def _ext():
    """The thin PyTorch extension (sv_torch, built beside the C-ABI library by
    build.py): the hot entry points take tensors through it.  Raises if it is
    missing; there is no other path."""
    if not _EXT:
        import importlib
        try:
            _EXT.append(importlib.import_module(__package__ + ".sv_torch"))
        except ImportError as e:
            raise RuntimeError("the sv_torch extension is not built (run comfyui-starvector-gguf_b200/build.py)") \
                from e
    return _EXT[0]


def _history(rows, vocab, history=None, history_len=None, seen=None, seen_bits=None):
    """(pointer, kind, row stride, len pointer, cols, keep-alive) for one history form."""
    t, kind, stride, lens, cols = _history_t(rows, vocab, history, history_len, seen, seen_bits)
    return _ptr(t), kind, stride, _ptr(lens), cols, (t, lens)


def _history_t(rows, vocab, history=None, history_len=None, seen=None, seen_bits=None):
    """(tensor, kind, row stride, lengths tensor, cols) for one history form."""
    if sum(x is not None for x in (history, seen, seen_bits)) > 1:
        raise ValueError("pass at most one of history, seen, seen_bits")
    if history is not None:
        _need_cuda(history, "history")
        h = history if history.dim() == 2 else history.unsqueeze(0)
        if h.dtype not in (torch.int32, torch.int64):
            raise ValueError("history ids must be int32 or int64")
        if h.stride(-1) != 1:
            h = h.contiguous()
        kind = L.HIST_IDS32 if h.dtype == torch.int32 else L.HIST_IDS64
        stride = h.stride(0) if h.shape[0] > 1 else 0
        lens = None
        if history_len is not None:
            lens = history_len.to(device=h.device, dtype=torch.int32).contiguous()
        return h, kind, stride, lens, h.shape[1]
    if seen is not None:
        _need_cuda(seen, "seen")
        s = seen if seen.dim() == 2 else seen.unsqueeze(0)
        if s.dtype not in (torch.bool, torch.uint8):
            raise ValueError("seen must be bool or uint8")
        if s.stride(-1) != 1:
            s = s.contiguous()
        stride = s.stride(0) if s.shape[0] > 1 else 0
        return s, L.HIST_MASK8, stride, None, 0
    if seen_bits is not None:
        _need_cuda(seen_bits, "seen_bits")
        b = seen_bits if seen_bits.dim() == 2 else seen_bits.unsqueeze(0)
        if b.dtype != torch.int32 or b.stride(-1) != 1:
            raise ValueError("seen_bits must be a contiguous int32 bitmap [rows, ceil(vocab/32)]")
        stride = b.stride(0) if b.shape[0] > 1 else 0
        return b, L.HIST_BITS32, stride, None, 0
    return None, L.HIST_NONE, 0, None, 0


def seen_bitmap(rows, vocab, device):
    """An all-clear packed seen bitmap [rows, ceil(vocab/32)] (int32 storage)."""
    return torch.zeros((rows, (vocab + 31) // 32), dtype=torch.int32, device=device)


def sample_step(logits, uniforms, *, history=None, history_len=None, seen=None, seen_bits=None,
                temperature=1.5, top_p=0.9, top_k=50, keep=1, repetition_penalty=3.1, out_capacity=0,
                dense=None, update_seen_bits=None, force_general=False, path=None, out=None,
                test_wait_timeout=False):
    """Fused penalty + temperature + top-k + top-p + softmax + draw for each row.

    Mirrors runtime_shared.py:200-202 per row (see include/starvector_sampling.h).
    Returns a dict: token int64 [R], count int32 [R], status int32 [R], and when
    requested idx/prob/score [R, out_capacity] (kept tokens in index order) and
    dense [R, V] ('scores' = the _warp output, 'probs' = its softmax).
    path: None (automatic), 'stream' or 'cluster' selects the kernel.
    test_wait_timeout: test hook (SV_FLAG_TEST_WAIT_TIMEOUT): the streaming kernel's
    history-copy wait runs out and the rows report SV_ST_TIMEOUT.
    """
    x = _rows(logits)
    R, V = x.shape
    dev = x.device
    _need_cuda(uniforms, "uniforms")
    u = uniforms.reshape(-1)
    if u.dtype != torch.float32 or not u.is_contiguous() or u.numel() < R:
        raise ValueError("uniforms must be a contiguous float32 tensor with one value per row")
    ht, hk, hs, hl, hc = _history_t(R, V, history, history_len, seen, seen_bits)
    o = out if out is not None else {}  # filled in place: callers may preallocate
    if "token" not in o:
        o["token"] = torch.empty(R, dtype=torch.int64, device=dev)
    if "count" not in o:
        o["count"] = torch.empty(R, dtype=torch.int32, device=dev)
    if "status" not in o:
        o["status"] = torch.empty(R, dtype=torch.int32, device=dev)
    if out_capacity and "idx" not in o:
        o["idx"] = torch.full((R, out_capacity), -1, dtype=torch.int32, device=dev)
        o["prob"] = torch.zeros((R, out_capacity), dtype=torch.float32, device=dev)
        o["score"] = torch.zeros((R, out_capacity), dtype=torch.float32, device=dev)
    mode = {None: L.DENSE_NONE, "scores": L.DENSE_SCORES, "probs": L.DENSE_PROBS}[dense]
    if mode != L.DENSE_NONE and "dense" not in o:
        o["dense"] = torch.empty((R, V), dtype=torch.float32, device=dev)
    upd = update_seen_bits
    if upd is not None:
        _need_cuda(upd, "update_seen_bits")
    rc = _ext().sample_step(
        x, R, V, x.stride(0) if R > 1 else 0, ht, hk, hs, hl, hc, u, float(temperature), float(top_p), int(top_k),
        int(keep), float(repetition_penalty), o["token"], o["count"], o.get("idx"), o.get("prob"), o.get("score"),
        int(out_capacity), o.get("dense"), mode, V, o["status"],
        upd, 0 if upd is None else (upd.stride(0) if upd.dim() == 2 else upd.shape[-1]),
        (L.FLAG_FORCE_GENERAL if force_general else 0) | (L.FLAG_TEST_WAIT_TIMEOUT if test_wait_timeout else 0)
        | {None: 0, "cluster": L.FLAG_CLUSTER, "stream": L.FLAG_STREAM}[path])
    L.check(rc, "sv_sample_step")
    return o


_WORKSPACES = {}


def beam_workspace(beams, vocab, device):
    """A zero-filled workspace for sv_beam_step, cached per (device, stream, shape).

    Calls that overlap on the GPU must not share a workspace; the cache keys on the
    current stream for that reason."""
    device = torch.device(device)
    key = (device.index, _stream(device), beams, vocab)
    ws = _WORKSPACES.get(key)
    if ws is None:
        nbytes = L.lib().sv_beam_workspace_bytes(int(beams), int(vocab))
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def beam_step(logits, running_scores, uniforms, *, history=None, history_len=None, seen=None, seen_bits=None,
              temperature=1.5, top_p=0.9, top_k=50, keep=2, repetition_penalty=3.1, num_picks=None,
              out_capacity=0, dense_logprob=False, force_general=False, workspace=None, out=None):
    """One beam-sampling step (runtime_shared.py:230-237); see include/starvector_sampling.h.

    Returns a dict: picks int64 [P] (flattened beam*V + token), scores float [P],
    n int32 [1] (valid picks), status int32 [1]; optionally per-beam kept lists
    kept_count/kept_idx/kept_logprob/kept_prob and dense logprob [B, V].
    """
    x = _rows(logits)
    B, V = x.shape
    dev = x.device
    P = 2 * B if num_picks is None else int(num_picks)
    rs = running_scores.reshape(-1)
    _need_cuda(rs, "running_scores")
    if rs.dtype != torch.float32 or not rs.is_contiguous() or rs.numel() != B:
        raise ValueError("running_scores must be a contiguous float32 tensor [beams]")
    u = uniforms.reshape(-1)
    _need_cuda(u, "uniforms")
    if u.dtype != torch.float32 or not u.is_contiguous() or u.numel() < P:
        raise ValueError("uniforms must be a contiguous float32 tensor with num_picks values")
    ht, hk, hs, hl, hc = _history_t(B, V, history, history_len, seen, seen_bits)
    o = out if out is not None else {}  # filled in place: callers may preallocate
    # Only missing outputs are allocated (a preallocated dict costs no kernels).
    need = {"picks": lambda: torch.full((P,), -1, dtype=torch.int64, device=dev),
            "scores": lambda: torch.zeros(P, dtype=torch.float32, device=dev),
            "n": lambda: torch.zeros(1, dtype=torch.int32, device=dev),
            "status": lambda: torch.zeros(1, dtype=torch.int32, device=dev)}
    if out_capacity:
        need.update(kept_count=lambda: torch.zeros(B, dtype=torch.int32, device=dev),
                    kept_idx=lambda: torch.full((B, out_capacity), -1, dtype=torch.int32, device=dev),
                    kept_logprob=lambda: torch.zeros((B, out_capacity), dtype=torch.float32, device=dev),
                    kept_prob=lambda: torch.zeros((B, out_capacity), dtype=torch.float32, device=dev))
    if dense_logprob:
        need["dense_logprob"] = lambda: torch.empty((B, V), dtype=torch.float32, device=dev)
    for k, make in need.items():
        if k not in o:
            o[k] = make()
    ws = workspace if workspace is not None else beam_workspace(B, V, dev)
    rc = _ext().beam_step(
        x, B, V, x.stride(0) if B > 1 else 0, ht, hk, hs, hl, hc, rs, u, P, float(temperature), float(top_p),
        int(top_k), int(keep), float(repetition_penalty), o["picks"], o["scores"], o["n"], o["status"],
        o.get("kept_count"), o.get("kept_idx"), o.get("kept_logprob"), o.get("kept_prob"), int(out_capacity),
        o.get("dense_logprob"), V, ws, L.FLAG_FORCE_GENERAL if force_general else 0)
    L.check(rc, "sv_beam_step")
    return o


def loop_guard(tokens, lengths=None, window=64, repeats=3, out=None):
    """Loop-guard verdicts (bool [R]) for token rows [R, L] (runtime_shared.py:156-167)."""
    _need_cuda(tokens, "tokens")
    t = tokens if tokens.dim() == 2 else tokens.unsqueeze(0)
    if t.dtype not in (torch.int32, torch.int64):
        raise ValueError("tokens must be int32 or int64")
    if t.stride(-1) != 1 or (t.shape[0] > 1 and t.stride(0) != t.shape[1]):
        t = t.contiguous()  # the kernel may read each row's whole stride
    R, Lmax = t.shape
    if lengths is None:
        lengths = torch.full((R,), Lmax, dtype=torch.int32, device=t.device)
    ln = lengths.to(device=t.device, dtype=torch.int32).contiguous()
    v = out if out is not None else torch.empty(R, dtype=torch.uint8, device=t.device)
    # A single row passes its own length as the stride (the batched kernel then
    # splits it across a cluster).
    rc = _ext().loop_guard(t, R, t.stride(0) if R > 1 else Lmax, ln, int(window), int(repeats), v)
    L.check(rc, "sv_loop_guard")
    return v.bool() if out is None else v


def penalize(logits, seen=None, seen_bits=None, repetition_penalty=3.1):
    """The reference's _penalize (runtime_shared.py:170-173) as float32 [R, V]."""
    x = _rows(logits)
    R, V = x.shape
    hp, hk, hs, _, _, _keep = _history(R, V, None, None, seen, seen_bits)
    if hk == L.HIST_NONE:
        raise ValueError("penalize needs seen or seen_bits")
    out = torch.empty((R, V), dtype=torch.float32, device=x.device)
    rc = L.lib().sv_penalize(x.data_ptr(), _DTYPES[x.dtype], R, V, x.stride(0) if R > 1 else 0, hp, hk, hs,
                             float(repetition_penalty), out.data_ptr(), V, _stream(x.device))
    L.check(rc, "sv_penalize")
    return out


def seen_update(seen_bits, tokens, vocab):
    """seen[r, tokens[r]] = True on a packed bitmap."""
    t = tokens.reshape(-1).to(torch.int64).contiguous()
    rc = L.lib().sv_seen_update(seen_bits.data_ptr(), seen_bits.shape[0], seen_bits.stride(0), t.data_ptr(),
                                int(vocab), _stream(seen_bits.device))
    L.check(rc, "sv_seen_update")


def seen_reorder(src, dst, parents, tokens, vocab):
    """dst[b] = src[parents[b]] with bit tokens[b] set (runtime_shared.py:258-259)."""
    p = parents.reshape(-1).to(torch.int64).contiguous()
    t = None if tokens is None else tokens.reshape(-1).to(torch.int64).contiguous()
    rc = L.lib().sv_seen_reorder(src.data_ptr(), dst.data_ptr(), src.shape[0], int(vocab), src.stride(0),
                                 p.data_ptr(), _ptr(t), _stream(src.device))
    L.check(rc, "sv_seen_reorder")


def beam_advance(step_out, *, beams, vocab, step, last, stop_ids, eos_id, tails_in, tails_out, running_out,
                 parents_out, tokens_out, seen_in=None, seen_out=None, hist_in=None, hist_out=None,
                 whash_in=None, whash_out=None, guard_table=None, window=64):
    """The beam loop's next-step decision on the device (sv_beam_advance,
    runtime_shared.py:237-259): from one beam_step's outputs `step_out` (picks,
    scores, n, status) writes the next running scores, the chosen parents and
    tokens, the rows' advanced stop-id tails and (optionally) the reordered seen
    bitmaps, token histories and rolling window hashes (entering each row's window
    in the incremental loop guard's `guard_table`).  stop_ids: int64 [S] on the
    device (S <= 16); tails int64 [beams, S]; hist int32 [beams, capacity > step];
    whash int32 [beams]; eos_id None never matches."""
    picks, scores = step_out["picks"], step_out["scores"]
    _need_cuda(picks, "picks")
    S = stop_ids.numel() if stop_ids is not None else 0
    words = (int(vocab) + 31) // 32
    rc = _ext().beam_advance(
        picks, scores, step_out["n"], step_out["status"], int(beams), int(vocab), int(step), bool(last),
        stop_ids if S else None, -1 if eos_id is None else int(eos_id), tails_in if S else None,
        tails_out if S else None, running_out, parents_out, tokens_out, seen_in, seen_out,
        seen_in.stride(0) if seen_in is not None else words, hist_in, hist_out,
        hist_in.stride(0) if hist_in is not None else 0, whash_in, whash_out, guard_table, int(window))
    L.check(rc, "sv_beam_advance")


def guard_table(windows, device):
    """An empty occurrence table for the incremental loop guard with room for
    `windows` window entries (a power of two >= 2 x windows, all bits set)."""
    n = 64
    while n < 2 * windows:
        n *= 2
    return torch.full((n,), -1, dtype=torch.int64, device=device)


def loop_guard_incremental(table, tokens, insert_from, length, window=64, repeats=3, out=None, status=None):
    """Incremental loop guard (sv_loop_guard_incremental, runtime_shared.py:156-167):
    enters the windows of `tokens` (a CUDA int32/int64 row) ending at positions
    [insert_from, length) into `table`, then writes the verdict for the first
    `length` tokens to `out` (uint8 [1]); returns `out`."""
    _need_cuda(tokens, "tokens")
    t = tokens.reshape(-1)
    if t.dtype not in (torch.int32, torch.int64) or t.stride(0) != 1:
        raise ValueError("tokens must be a contiguous int32 or int64 row")
    if not 0 <= int(insert_from) <= int(length) <= t.numel():
        raise ValueError("need 0 <= insert_from <= length <= len(tokens)")
    if table.dtype != torch.int64 or not table.is_contiguous():
        raise ValueError("table must be a contiguous int64 tensor (guard_table)")
    v = out if out is not None else torch.empty(1, dtype=torch.uint8, device=t.device)
    rc = _ext().loop_guard_incremental(table, t, int(insert_from), int(length), int(window), int(repeats), v,
                                       status)
    L.check(rc, "sv_loop_guard_incremental")
    return v


def block_len(rows, capacity):
    """int32 values of one rank's slice block (the sv_merge_slices layout)."""
    return 2 * rows * capacity + 2 * rows


def slice_block_outputs(block, rows, capacity):
    """sample_step's `out` dict over one slice block int32 [block_len]: the slice
    step writes its scores, slice-local ids, counts and statuses straight into the
    exchange layout (the token goes to a separate int64 [rows])."""
    RC = rows * capacity
    return {"score": block[:RC].view(torch.float32).view(rows, capacity),
            "idx": block[RC:2 * RC].view(rows, capacity),
            "count": block[2 * RC:2 * RC + rows],
            "status": block[2 * RC + rows:2 * RC + 2 * rows],
            "token": torch.empty(rows, dtype=torch.int64, device=block.device)}


def merge_shards(packed, uniforms, *, capacity, top_p=0.9, top_k=50, keep=1, out_capacity=0, out=None,
                 rows=None, slice_stride=None):
    """Merges the all-gathered per-slice kept lists of a vocab-sharded sample step:
    records int32 [shards, rows, 2 * capacity + 2] (sv_merge_shards), or with
    slice_stride given, slice blocks int32 [shards, block_len(rows, capacity)]
    (sv_merge_slices).

    Returns a dict: token int64 [rows], count int32 [rows], status int32 [rows],
    and idx / prob [rows, out_capacity] when out_capacity > 0.
    """
    _need_cuda(packed, "packed")
    blocked = slice_stride is not None
    if blocked:
        if packed.dtype != torch.int32 or packed.dim() != 2 or not packed.is_contiguous() or rows is None or \
                packed.shape[1] != block_len(rows, capacity):
            raise ValueError("blocks must be a contiguous int32 tensor [shards, 2 rows capacity + 2 rows]")
        S, R = packed.shape[0], int(rows)
    else:
        if packed.dtype != torch.int32 or packed.dim() != 3 or not packed.is_contiguous():
            raise ValueError("packed must be a contiguous int32 tensor [shards, rows, 2 * capacity + 2]")
        S, R, W = packed.shape
        if W != 2 * capacity + 2:
            raise ValueError("packed records must hold 2 * capacity + 2 values")
    u = uniforms.reshape(-1)
    _need_cuda(u, "uniforms")
    if u.dtype != torch.float32 or not u.is_contiguous() or u.numel() < R:
        raise ValueError("uniforms must be a contiguous float32 tensor with one value per row")
    dev = packed.device
    o = out if out is not None else {}
    need = {"token": lambda: torch.empty(R, dtype=torch.int64, device=dev),
            "count": lambda: torch.empty(R, dtype=torch.int32, device=dev),
            "status": lambda: torch.empty(R, dtype=torch.int32, device=dev)}
    if out_capacity:
        need.update(idx=lambda: torch.full((R, out_capacity), -1, dtype=torch.int32, device=dev),
                    prob=lambda: torch.zeros((R, out_capacity), dtype=torch.float32, device=dev))
    for k, make in need.items():
        if k not in o:
            o[k] = make()
    if blocked:
        rc = L.lib().sv_merge_slices(packed.data_ptr(), S, R, int(capacity), int(slice_stride), u.data_ptr(),
                                     float(top_p), int(top_k), int(keep), o["token"].data_ptr(),
                                     o["count"].data_ptr(), _ptr(o.get("idx")), _ptr(o.get("prob")),
                                     int(out_capacity), o["status"].data_ptr(), _stream(dev))
        L.check(rc, "sv_merge_slices")
    else:
        rc = L.lib().sv_merge_shards(packed.data_ptr(), S, R, int(capacity), u.data_ptr(), float(top_p), int(top_k),
                                     int(keep), o["token"].data_ptr(), o["count"].data_ptr(), _ptr(o.get("idx")),
                                     _ptr(o.get("prob")), int(out_capacity), o["status"].data_ptr(), _stream(dev))
        L.check(rc, "sv_merge_shards")
    return o


def pack_slice(local, offset, capacity, out):
    """A rank's exchange records (sv_pack_slice) from its slice step's outputs
    (count, status, idx, score [rows, capacity]) into out int32 [rows, 2C + 2]."""
    for k in ("count", "status", "idx", "score"):
        _need_cuda(local[k], k)
    R = local["count"].shape[0]
    if tuple(local["idx"].shape) != (R, capacity) or not out.is_contiguous():
        raise ValueError("slice outputs must have capacity columns and the records be contiguous")
    rc = L.lib().sv_pack_slice(local["count"].data_ptr(), local["status"].data_ptr(), local["idx"].data_ptr(),
                               local["score"].data_ptr(), R, int(capacity), int(offset), out.data_ptr(),
                               _stream(out.device))
    L.check(rc, "sv_pack_slice")
    return out


def beam_slice_stats(logits_slice, global_max=None, out=None):
    """One rank's slice statistics for the vocab-sharded beam step
    (sv_beam_slice_stats).  Without global_max: {"max": float [beams], "flags":
    int32 [beams]} (2 NaN, 1 +inf, 0 neither), to all-reduce with MAX.  With the
    reduced maxima: {"sum": int64 [beams]}, the exact fixed-point exp sums, to
    all-reduce with SUM.  `out` may hold those tensors already (filled in place)."""
    x = _rows(logits_slice)
    B, W = x.shape
    dev = x.device
    stride = x.stride(0) if B > 1 else 0
    o = out if out is not None else {}
    if global_max is None:
        mx = o.get("max")
        mx = mx if mx is not None else torch.empty(B, dtype=torch.float32, device=dev)
        fl = o.get("flags")
        fl = fl if fl is not None else torch.empty(B, dtype=torch.int32, device=dev)
        rc = L.lib().sv_beam_slice_stats(x.data_ptr(), _DTYPES[x.dtype], B, W, stride, None, mx.data_ptr(),
                                         fl.data_ptr(), None, _stream(dev))
        L.check(rc, "sv_beam_slice_stats")
        return {"max": mx, "flags": fl}
    gm = global_max.reshape(-1)
    _need_cuda(gm, "global_max")
    if gm.dtype != torch.float32 or not gm.is_contiguous() or gm.numel() != B:
        raise ValueError("global_max must be a contiguous float32 tensor [beams]")
    sm = o.get("sum")
    sm = sm if sm is not None else torch.empty(B, dtype=torch.int64, device=dev)
    rc = L.lib().sv_beam_slice_stats(x.data_ptr(), _DTYPES[x.dtype], B, W, stride, gm.data_ptr(), None, None,
                                     sm.data_ptr(), _stream(dev))
    L.check(rc, "sv_beam_slice_stats")
    return {"sum": sm}


def beam_slice_logprobs(logits_slice, global_max, global_sum, out=None):
    """The slice's log_softmax (x - M) - ln(S 2^-44), float32 [beams, width], from the
    all-reduced statistics (sv_beam_slice_logprobs)."""
    x = _rows(logits_slice)
    B, W = x.shape
    dev = x.device
    gm, gs = global_max.reshape(-1), global_sum.reshape(-1)
    for t, n, dt in ((gm, "global_max", torch.float32), (gs, "global_sum", torch.int64)):
        _need_cuda(t, n)
        if t.dtype != dt or not t.is_contiguous() or t.numel() != B:
            raise ValueError(f"{n} must be a contiguous {dt} tensor [beams]")
    o = out if out is not None else torch.empty((B, W), dtype=torch.float32, device=dev)
    rc = L.lib().sv_beam_slice_logprobs(x.data_ptr(), _DTYPES[x.dtype], B, W, x.stride(0) if B > 1 else 0,
                                        gm.data_ptr(), gs.data_ptr(), o.data_ptr(), o.stride(0) if B > 1 else 0,
                                        _stream(dev))
    L.check(rc, "sv_beam_slice_logprobs")
    return o


def merge_beam_shards(packed, global_max, global_flags, running_scores, uniforms, *, capacity, vocab, top_p=0.9,
                      top_k=50, keep=2, num_picks=None, out_capacity=0, workspace=None, out=None, beams=None,
                      slice_stride=None):
    """Merge side of the vocab-sharded beam step: records int32 [shards, beams,
    2 * capacity + 2] (sv_merge_beam_shards), or with slice_stride given, slice
    blocks int32 [shards, block_len(beams, capacity)] (sv_merge_beam_slices).
    Returns beam_step's dict (picks, scores, n, status, and the per-beam kept lists
    when out_capacity > 0)."""
    _need_cuda(packed, "packed")
    blocked = slice_stride is not None
    if blocked:
        if packed.dtype != torch.int32 or packed.dim() != 2 or not packed.is_contiguous() or beams is None or \
                packed.shape[1] != block_len(beams, capacity):
            raise ValueError("blocks must be a contiguous int32 tensor [shards, 2 beams capacity + 2 beams]")
        S, B = packed.shape[0], int(beams)
    else:
        if packed.dtype != torch.int32 or packed.dim() != 3 or not packed.is_contiguous():
            raise ValueError("packed must be a contiguous int32 tensor [shards, beams, 2 * capacity + 2]")
        S, B, Wd = packed.shape
        if Wd != 2 * capacity + 2:
            raise ValueError("packed records must hold 2 * capacity + 2 values")
    P = 2 * B if num_picks is None else int(num_picks)
    dev = packed.device
    rs, u = running_scores.reshape(-1), uniforms.reshape(-1)
    for t, n, size in ((rs, "running_scores", B), (u, "uniforms", P)):
        _need_cuda(t, n)
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < size:
            raise ValueError(f"{n} must be a contiguous float32 tensor with {size} values")
    gm, gf = global_max.reshape(-1), global_flags.reshape(-1)
    if gm.dtype != torch.float32 or gf.dtype != torch.int32 or gm.numel() != B or gf.numel() != B:
        raise ValueError("global_max float32 [beams] and global_flags int32 [beams]")
    o = out if out is not None else {}
    need = {"picks": lambda: torch.full((P,), -1, dtype=torch.int64, device=dev),
            "scores": lambda: torch.zeros(P, dtype=torch.float32, device=dev),
            "n": lambda: torch.zeros(1, dtype=torch.int32, device=dev),
            "status": lambda: torch.zeros(1, dtype=torch.int32, device=dev)}
    if out_capacity:
        need.update(kept_count=lambda: torch.zeros(B, dtype=torch.int32, device=dev),
                    kept_idx=lambda: torch.full((B, out_capacity), -1, dtype=torch.int32, device=dev),
                    kept_logprob=lambda: torch.zeros((B, out_capacity), dtype=torch.float32, device=dev),
                    kept_prob=lambda: torch.zeros((B, out_capacity), dtype=torch.float32, device=dev))
    for k, make in need.items():
        if k not in o:
            o[k] = make()
    ws = workspace
    if ws is None:
        key = ("merge_beam", dev.index, _stream(dev), B, S, int(capacity))
        ws = _WORKSPACES.get(key)
        if ws is None:
            nbytes = L.lib().sv_merge_beam_shards_workspace_bytes(B, S, int(capacity))
            ws = _WORKSPACES[key] = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    tail = (gm.data_ptr(), gf.data_ptr(), rs.data_ptr(), u.data_ptr(), P, float(top_p), int(top_k), int(keep),
            ws.data_ptr(), ws.numel(), o["picks"].data_ptr(), o["scores"].data_ptr(), o["n"].data_ptr(),
            o["status"].data_ptr(), _ptr(o.get("kept_count")), _ptr(o.get("kept_idx")), _ptr(o.get("kept_logprob")),
            _ptr(o.get("kept_prob")), int(out_capacity), _stream(dev))
    if blocked:
        rc = L.lib().sv_merge_beam_slices(packed.data_ptr(), S, B, int(capacity), int(slice_stride), int(vocab),
                                          *tail)
        L.check(rc, "sv_merge_beam_slices")
    else:
        rc = L.lib().sv_merge_beam_shards(packed.data_ptr(), S, B, int(capacity), int(vocab), *tail)
        L.check(rc, "sv_merge_beam_shards")
    return o


def kv_reorder(keys, values, parents, length, out_status=None):
    """The beam step's KV-cache reorder in place (sv_kv_reorder,
    runtime_shared.py:388-394): rows whose parent changed receive the parent's
    first `length` slots.  keys / values: [layers, beams, capacity, head_dim] (MQA)
    or [layers, beams, heads, capacity, head_dim] (GQA), the same layout each
    (values may be None); parents: int64 [beams] on the device."""
    _need_cuda(keys, "keys")
    if keys.dim() == 4:
        Lr, B, cap, D = keys.shape
        H, sl, sb, sh, ss = 1, keys.stride(0), keys.stride(1), 0, keys.stride(2)
    elif keys.dim() == 5:
        Lr, B, H, cap, D = keys.shape
        sl, sb, sh, ss = keys.stride(0), keys.stride(1), keys.stride(2), keys.stride(3)
    else:
        raise ValueError("keys must be [layers, beams, capacity, head_dim] or [layers, beams, heads, capacity, "
                         "head_dim]")
    if keys.stride(-1) != 1:
        raise ValueError("head_dim must be contiguous")
    if values is not None and (values.shape != keys.shape or values.stride() != keys.stride() or
                               values.dtype != keys.dtype):
        raise ValueError("values must have the keys' shape, strides and dtype")
    if not 0 <= int(length) <= cap:
        raise ValueError("length must be in [0, capacity]")
    p = parents.reshape(-1)
    _need_cuda(p, "parents")
    if p.dtype != torch.int64 or not p.is_contiguous() or p.numel() != B:
        raise ValueError("parents must be a contiguous int64 tensor [beams]")
    rc = _ext().kv_reorder(keys, values, Lr, B, H, int(length), D, sl, sb, sh, ss, p, out_status)
    L.check(rc, "sv_kv_reorder")
