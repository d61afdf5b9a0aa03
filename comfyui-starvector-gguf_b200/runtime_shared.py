"""Drop-in for the sampling step of ComfyUI-StarVector-GGUF's runtime_shared.py.

Same names, arguments, return values and errors as the reference's sampling
functions (runtime_shared.py:147-265): the constants, `_repeating`, `_penalize`,
`_warp`, `_ends`, `_sample` and `_beam_sample`.  The reference's own
`generate_tokens` (:268-342) stays in use: it calls `_sample` / `_beam_sample`
through its module's globals, and `install(module)` rebinds those names (and
`_repeating`, `_penalize`, `_warp`) to the functions here.  The decoder protocol is
unchanged (`prefill(embeddings, rows, capacity)` returning a decoding object with
`step(tokens)` / `reorder(parents)` plus the first logits).

What changes is where the per-token sampling step runs: one fused sm_100a kernel
per step (penalty from an on-device seen bitmap, temperature, top-k, top-p,
softmax, draw, seen update), the beam step in one launch, and the loop guard on a
device-resident token history.  Draws come from uniforms generated on the device
from the same seed (`torch.manual_seed(seed)` inside `fork_rng`, as the reference);
the draw rule is an inverse CDF over the kept tokens, so the sampled distribution
equals torch.multinomial's while individual samples differ from the reference's
for the same seed.  Logits must live on a CUDA device.
"""
from __future__ import annotations

from array import array

import torch

from . import _lib as L
from . import ops

# Transformers' sampling settings of the StarVector quickstart (runtime_shared.py:147-153).
TOP_K = 50
REPETITION_PENALTY = 3.1
LENGTH_PENALTY = -1.0
LOOP_WINDOW = 64
LOOP_REPEATS = 3


def _raise_status(status: int) -> None:
    raise RuntimeError(f"probability tensor contains either `inf`, `nan` or element < 0 "
                       f"({L.error_string(status)})")


def _repeating(tokens, device=None):
    """True when the last LOOP_WINDOW tokens occur LOOP_REPEATS times (runtime_shared.py:156-167).

    `tokens` is a host list (as in the reference) or a CUDA int tensor [L]."""
    if isinstance(tokens, torch.Tensor):
        t = tokens.reshape(1, -1)
    else:
        if len(tokens) < LOOP_WINDOW * LOOP_REPEATS:
            return False
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        t = torch.tensor([list(tokens)], dtype=torch.int32, device=dev)
    if t.shape[1] < LOOP_WINDOW * LOOP_REPEATS:
        return False
    return bool(ops.loop_guard(t, window=LOOP_WINDOW, repeats=LOOP_REPEATS)[0])


def _penalize(scores, seen):
    """Transformers' RepetitionPenaltyLogitsProcessor over the generated tokens (:170-173)."""
    return ops.penalize(scores, seen=seen, repetition_penalty=REPETITION_PENALTY).reshape(scores.shape)


def _warp(scores, temperature, top_p, keep):
    """Transformers' temperature, top-k and top-p warpers, in that order (:176-187)."""
    x = scores.reshape(-1, scores.shape[-1])
    u = torch.zeros(x.shape[0], dtype=torch.float32, device=x.device)
    o = ops.sample_step(x, u, temperature=temperature, top_p=top_p, top_k=TOP_K, keep=keep,
                        repetition_penalty=REPETITION_PENALTY, dense="scores")
    status = o["status"].max().item()
    if status:
        _raise_status(int(status))
    return o["dense"].reshape(scores.shape)


def _ends(tokens, stop_ids, eos_id):
    return tokens[-1] == eos_id or tokens[-len(stop_ids):] == stop_ids


class _TokenHistory:
    """Device copy of each row's generated tokens (int64), for the loop guard.  The
    sampling kernel writes each step's token straight into its slot."""

    def __init__(self, rows, capacity, device):
        self.ids = torch.zeros((rows, max(capacity, 1)), dtype=torch.int64, device=device)

    def slot(self, step):
        """Row 0's slot of a step, as the kernel's token output."""
        return self.ids[0, step:step + 1]


# The host reads the sampled tokens once per loop-guard period (runtime_shared.py:207)
# instead of once per token.
_SYNC_EVERY = 16

_PINNED = {}


def _read_block(arrays, first, last, device):
    """Host lists of rows [first, last] of device arrays (a dict), through pinned
    buffers cached per shape and one stream synchronisation.  The buffers are shared
    by every generation of the process: one generation at a time (as ComfyUI runs
    its prompts)."""
    k = last + 1 - first
    host = {}
    for name, t in arrays.items():
        key = (name, t.dtype, tuple(t.shape[1:]))
        buf = _PINNED.get(key)
        if buf is None or buf.shape[0] < k:
            buf = _PINNED[key] = torch.empty((max(k, _SYNC_EVERY), *t.shape[1:]), dtype=t.dtype, pin_memory=True)
        buf[:k].copy_(t[first:last + 1], non_blocking=True)
        host[name] = buf
    torch.cuda.current_stream(device).synchronize()
    return {name: buf[:k].tolist() for name, buf in host.items()}


def _sample(decoder, embeddings, max_new_tokens, temperature, top_p, stop_ids, eos_id, loop_guard, on_step,
            uniforms=None):
    """Transformers' multinomial sampling of one sequence (runtime_shared.py:194-211).

    The tokens stay on the device: the host reads them (and the steps' statuses and
    loop-guard verdicts) once every 16 steps and at the last step, then goes through
    that block's steps in order - the status check, the progress callback, the end
    check and, every 16th step, the loop guard - exactly as the reference does per
    token, so the tokens, the stop reason, the callbacks and the errors are the
    reference's.  The loop guard is incremental (sv_loop_guard_incremental): each
    check enters the 16 new windows in an occurrence table and probes it for the
    tail, in time independent of the sequence's length.  Up to 15 decode steps
    issued after an end inside a block are discarded.
    """
    decoding, logits = decoder.prefill(embeddings, 1, embeddings.shape[1] + max_new_tokens)
    device, vocab = logits.device, logits.shape[-1]
    if uniforms is None:
        uniforms = torch.rand((max_new_tokens, 1), dtype=torch.float32, device=device)
    seen = ops.seen_bitmap(1, vocab, device)
    history = _TokenHistory(1, max_new_tokens, device)
    statuses = torch.zeros(max_new_tokens, dtype=torch.int32, device=device)
    verdicts = torch.zeros(max_new_tokens, dtype=torch.uint8, device=device)
    table = ops.guard_table(max_new_tokens, device) if loop_guard else None
    guarded = 0  # tokens whose windows are in the table
    out = {}
    tokens = []
    synced = 0
    for step in range(max_new_tokens):
        # The kernel writes the token into the history and the status in place.
        out["token"] = history.slot(step)
        out["status"] = statuses[step:step + 1]
        out = ops.sample_step(logits.reshape(1, vocab), uniforms[step], seen_bits=seen, temperature=temperature,
                              top_p=top_p, top_k=TOP_K, keep=1, repetition_penalty=REPETITION_PENALTY,
                              update_seen_bits=seen, out=out)
        if loop_guard and step % 16 == 15:
            ops.loop_guard_incremental(table, history.ids[0], guarded, step + 1, LOOP_WINDOW, LOOP_REPEATS,
                                       out=verdicts[step:step + 1])
            guarded = step + 1
        if step % _SYNC_EVERY == _SYNC_EVERY - 1 or step + 1 == max_new_tokens:
            block = _read_block({"token": history.ids[0], "status": statuses, "verdict": verdicts}, synced, step,
                                device)
            for j, (value, status, verdict) in enumerate(zip(block["token"], block["status"], block["verdict"]),
                                                         start=synced):
                if value < 0:
                    _raise_status(int(status))
                tokens.append(value)
                on_step(j + 1)
                if _ends(tokens, stop_ids, eos_id):
                    return tokens, 'stop'
                if loop_guard and j % 16 == 15 and verdict:
                    return tokens, 'repetition'
            synced = step + 1
        if step + 1 < max_new_tokens:
            # A failed step's token is -1 until the host reads the block and raises;
            # the decoder is fed token 0 for it, so it only ever sees valid ids.
            logits = decoding.step(out["token"].clamp_min(0))
    return tokens, 'token_limit'


# Stop sequences up to this many tokens are matched on the device (sv_beam_advance).
_MAX_STOP = 16


def _node_tokens(node, limit=None):
    """The tokens of a candidate held as a linked node (token, parent node), oldest
    first; only the last `limit` when given."""
    out = []
    while node is not None and (limit is None or len(out) < limit):
        out.append(node[0])
        node = node[1]
    out.reverse()
    return out


def _node_ends(node, stop_ids, eos_id):
    """_ends (runtime_shared.py:190-191) of a candidate node: its last token is
    eos_id, or its last len(stop_ids) tokens equal stop_ids."""
    if node[0] == eos_id:
        return True
    return len(stop_ids) > 0 and _node_tokens(node, len(stop_ids)) == stop_ids


def _device_reorder(decoding, beams):
    """A function applying device-resident parents to the decoder's cache, or None
    when the decoder only takes host lists.  Decoders may offer
    `reorder_device(parents)`; the reference's own CachedDecoding
    (runtime_shared.py:388-394) is reordered by sv_kv_reorder on its keys and
    values, which is what its `reorder` does with torch indexing."""
    fn = getattr(decoding, "reorder_device", None)
    if callable(fn):
        return fn
    keys, values, length = (getattr(decoding, name, None) for name in ("keys", "values", "length"))
    if type(decoding).__name__ != "CachedDecoding" or not isinstance(length, int):
        return None
    if not (isinstance(keys, torch.Tensor) and isinstance(values, torch.Tensor) and keys.is_cuda
            and keys.dim() in (4, 5) and keys.shape[1] == beams):
        return None
    try:  # identity parents: checks the cache layout, copies nothing
        ops.kv_reorder(keys, values, torch.arange(beams, device=keys.device), length)
    except (ValueError, RuntimeError):
        return None
    return lambda parents: ops.kv_reorder(decoding.keys, decoding.values, parents, decoding.length)


class _BeamRecord:
    """Per-step device records of a beam generation: the beam step's picks, scores,
    pick count and status, the device's decision (running scores, parents, tokens)
    and the loop-guard verdicts."""

    def __init__(self, steps, beams, picks, device):
        self.picks = torch.full((steps, picks), -1, dtype=torch.int64, device=device)
        self.scores = torch.zeros((steps, picks), dtype=torch.float32, device=device)
        self.n = torch.zeros(steps, dtype=torch.int32, device=device)
        self.status = torch.zeros(steps, dtype=torch.int32, device=device)
        self.running = torch.zeros((steps + 1, beams), dtype=torch.float32, device=device)
        self.parents = torch.zeros((steps, beams), dtype=torch.int64, device=device)
        self.tokens = torch.zeros((steps, beams), dtype=torch.int64, device=device)
        self.verdict = torch.zeros(steps, dtype=torch.uint8, device=device)

    def step_out(self, step):
        return {"picks": self.picks[step], "scores": self.scores[step], "n": self.n[step:step + 1],
                "status": self.status[step:step + 1]}

    def read(self, first, last, device):
        """Host lists of steps [first, last] (running = the scores after each step)."""
        return _read_block({"picks": self.picks, "scores": self.scores, "n": self.n, "status": self.status,
                            "running": self.running[1:], "parents": self.parents, "tokens": self.tokens,
                            "verdict": self.verdict}, first, last, device)


def _beam_sample(decoder, embeddings, max_new_tokens, temperature, top_p, beams, stop_ids, eos_id, loop_guard,
                 on_step, uniforms=None):
    """Transformers' beam sampling with early_stopping=True for one prompt (runtime_shared.py:214-265).

    Each step samples 2 * beams continuations without replacement from all beams.
    Only the first `beams` samples may finish; the best unfinished samples continue.
    Finished scores use the length penalty.

    The step's decision - which candidates continue, their running scores, parents
    and tokens, the seen bitmaps and the rows' token histories - is taken on the
    device (sv_beam_advance), and the decoder's cache is reordered from the device
    parents, so no step waits for the host.  The host reads the steps' records once
    every 16 steps and replays the reference's bookkeeping over them in order (the
    finished list with the length penalty in float64, the stop tests, the progress
    callback, the loop guard), checking the device's decision step by step, so the
    result, stop reason, callbacks and errors are the reference's.  Up to 15 decode
    steps issued after an end inside a block are discarded.  A decoder whose cache
    can only be reordered from a host list is driven one step at a time.
    """
    keep = 2 * beams
    decoding, logits = decoder.prefill(embeddings, beams, embeddings.shape[1] + max_new_tokens)
    device, vocab = logits.device, logits.shape[-1]
    steps = max_new_tokens
    if uniforms is None:
        uniforms = torch.rand((steps, keep), dtype=torch.float32, device=device)
    # A stop list that is not a list never equals a list slice in the reference.
    n_stop = len(stop_ids) if isinstance(stop_ids, list) else 0
    if n_stop > _MAX_STOP:
        raise ValueError(f"stop sequences longer than {_MAX_STOP} tokens are not supported")
    reorder_cache = _device_reorder(decoding, beams)
    every = _SYNC_EVERY if reorder_cache is not None else 1
    rec = _BeamRecord(steps, beams, keep, device)
    rec.running[0, 1:] = -1e9
    stop_dev = torch.tensor(stop_ids, dtype=torch.int64, device=device) if n_stop else None
    tails = torch.full((2, beams, max(n_stop, 1)), -1, dtype=torch.int64, device=device)
    seen = (ops.seen_bitmap(beams, vocab, device), ops.seen_bitmap(beams, vocab, device))
    hist = torch.zeros((2, beams, steps), dtype=torch.int32, device=device) if loop_guard else None
    # The incremental loop guard: every running row's window at every step enters
    # one occurrence table (inside sv_beam_advance); a check probes it for row 0.
    whash = torch.zeros((2, beams), dtype=torch.int32, device=device) if loop_guard else None
    table = ops.guard_table(beams * steps, device) if loop_guard else None
    workspace = ops.beam_workspace(beams, vocab, device)

    # The reference's host state, with candidates as linked nodes (token, parent).
    running = [None] * beams
    finished = []
    improvable = True

    def result(reason=None):
        if reason == 'repetition':
            return _node_tokens(finished[0][1] if finished else running[0]), reason
        if not finished:
            return _node_tokens(running[0]), 'token_limit'
        best = _node_tokens(finished[0][1])
        return best, ('token_limit' if len(best) == steps and not _ends(best, stop_ids, eos_id) else 'stop')

    def replay(first, last_step):
        """The reference's bookkeeping (runtime_shared.py:237-256) over steps
        [first, last_step]; returns (result or None, the last step's parents)."""
        nonlocal running, finished, improvable
        h = rec.read(first, last_step, device)
        selected = None
        for k, step in enumerate(range(first, last_step + 1)):
            n, status = h["n"][k], h["status"][k]
            if status:
                _raise_status(status)
            picked = h["scores"][k][:n]
            parents, tokens = zip(*(divmod(pick, vocab) for pick in h["picks"][k][:n]))
            candidates = [(token, running[parent]) for parent, token in zip(parents, tokens)]
            last = step + 1 == steps
            hits = [last or _node_ends(candidate, stop_ids, eos_id) for candidate in candidates]
            if improvable and len(finished) < beams:
                finished += [(picked[j] / (step + 1) ** LENGTH_PENALTY, candidates[j])
                             for j in range(min(beams, len(picked))) if hits[j]]
                finished = sorted(finished, key=lambda item: item[0], reverse=True)[:beams]
            live = [score - 1e9 * hit for score, hit in zip(picked, hits)]
            order = sorted(range(len(picked)), key=live.__getitem__, reverse=True)[:beams]
            running_scores = [live[j] for j in order] + [-1e9] * (beams - len(order))
            order += [order[0]] * (beams - len(order))
            running = [candidates[j] for j in order]
            selected = [parents[j] for j in order]
            if (selected != h["parents"][k] or [tokens[j] for j in order] != h["tokens"][k]
                    or array('f', running_scores).tolist() != h["running"][k]):
                raise RuntimeError(f"beam step {step}: the device's decision differs from the host replay")
            on_step(step + 1)
            worst = min(score for score, _ in finished) if len(finished) == beams else -1e9
            improvable = improvable and running_scores[0] / (step + 1) ** LENGTH_PENALTY > worst
            if not improvable or len(finished) == beams or all(hits):
                return result(), selected
            if loop_guard and step % 16 == 15 and h["verdict"][k]:
                return result('repetition'), selected
        return None, selected

    synced = 0
    for step in range(steps):
        cur, nxt = step % 2, 1 - step % 2
        out = rec.step_out(step)
        ops.beam_step(logits.reshape(-1, vocab), rec.running[step], uniforms[step], seen_bits=seen[cur],
                      temperature=temperature, top_p=top_p, top_k=TOP_K, keep=2,
                      repetition_penalty=REPETITION_PENALTY, num_picks=keep, workspace=workspace, out=out)
        last = step + 1 == steps
        ops.beam_advance(out, beams=beams, vocab=vocab, step=step, last=last, stop_ids=stop_dev, eos_id=eos_id,
                         tails_in=tails[cur], tails_out=tails[nxt], running_out=rec.running[step + 1],
                         parents_out=rec.parents[step], tokens_out=rec.tokens[step], seen_in=seen[cur],
                         seen_out=seen[nxt], hist_in=None if hist is None else hist[cur],
                         hist_out=None if hist is None else hist[nxt],
                         whash_in=None if whash is None else whash[cur],
                         whash_out=None if whash is None else whash[nxt], guard_table=table, window=LOOP_WINDOW)
        if loop_guard and step % 16 == 15:
            # running[0]'s tokens after this step (runtime_shared.py:254).
            ops.loop_guard_incremental(table, hist[nxt, 0], step + 1, step + 1, LOOP_WINDOW, LOOP_REPEATS,
                                       out=rec.verdict[step:step + 1])
        if step % every == every - 1 or last:
            done, selected = replay(synced, step)
            if done is not None:
                return done
            synced = step + 1
        if not last:
            if reorder_cache is not None:
                reorder_cache(rec.parents[step])
            else:
                decoding.reorder(selected)
            logits = decoding.step(rec.tokens[step])
    raise AssertionError("the last step always ends the loop")  # every candidate hits at the last step


def install(module) -> None:
    """Rebind the reference module's sampling functions to these (its own
    `generate_tokens`, runtime_shared.py:268-342, then runs the kernels)."""
    for name in ("_repeating", "_penalize", "_warp", "_sample", "_beam_sample"):
        setattr(module, name, globals()[name])
