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
        self.length = 0

    def slot(self, step):
        """Row 0's slot of a step, as the kernel's token output."""
        return self.ids[0, step:step + 1]

    def repeating(self, row=0, length=None):
        length = self.length if length is None else length
        if length < LOOP_WINDOW * LOOP_REPEATS:
            return False
        lengths = torch.full((1,), length, dtype=torch.int32, device=self.ids.device)
        return bool(ops.loop_guard(self.ids[row:row + 1], lengths, LOOP_WINDOW, LOOP_REPEATS)[0])


# The host reads the sampled tokens once per loop-guard period (runtime_shared.py:207)
# instead of once per token.
_SYNC_EVERY = 16


def _sample(decoder, embeddings, max_new_tokens, temperature, top_p, stop_ids, eos_id, loop_guard, on_step,
            uniforms=None):
    """Transformers' multinomial sampling of one sequence (runtime_shared.py:194-211).

    The tokens stay on the device: the host reads them (and the steps' statuses) once
    every 16 steps and at the last step, then goes through that block's steps in
    order - the status check, the progress callback, the end check and, every 16th
    step, the loop guard - exactly as the reference does per token, so the tokens,
    the stop reason, the callbacks and the errors are the reference's.  Up to 15
    decode steps issued after an end inside a block are discarded.
    """
    decoding, logits = decoder.prefill(embeddings, 1, embeddings.shape[1] + max_new_tokens)
    device, vocab = logits.device, logits.shape[-1]
    if uniforms is None:
        uniforms = torch.rand((max_new_tokens, 1), dtype=torch.float32, device=device)
    seen = ops.seen_bitmap(1, vocab, device)
    history = _TokenHistory(1, max_new_tokens, device)
    statuses = torch.zeros(max_new_tokens, dtype=torch.int32, device=device)
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
        history.length = step + 1
        if step % _SYNC_EVERY == _SYNC_EVERY - 1 or step + 1 == max_new_tokens:
            block = history.ids[0, synced:step + 1].tolist()
            block_status = statuses[synced:step + 1].tolist()
            for j, (value, status) in enumerate(zip(block, block_status), start=synced):
                if value < 0:
                    _raise_status(int(status))
                tokens.append(value)
                on_step(j + 1)
                if _ends(tokens, stop_ids, eos_id):
                    return tokens, 'stop'
                if loop_guard and j % 16 == 15 and history.repeating(length=j + 1):
                    return tokens, 'repetition'
            synced = step + 1
        if step + 1 < max_new_tokens:
            # A failed step's token is -1 until the host reads the block and raises;
            # the decoder is fed token 0 for it, so it only ever sees valid ids.
            logits = decoding.step(out["token"].clamp_min(0))
    return tokens, 'token_limit'


def _beam_sample(decoder, embeddings, max_new_tokens, temperature, top_p, beams, stop_ids, eos_id, loop_guard,
                 on_step, uniforms=None):
    """Transformers' beam sampling with early_stopping=True for one prompt (runtime_shared.py:214-265).

    Each step samples 2 * beams continuations without replacement from all beams.
    Only the first `beams` samples may finish; the best unfinished samples continue.
    Finished scores use the length penalty.
    """
    keep = 2 * beams
    decoding, logits = decoder.prefill(embeddings, beams, embeddings.shape[1] + max_new_tokens)
    device, vocab = logits.device, logits.shape[-1]
    if uniforms is None:
        uniforms = torch.rand((max_new_tokens, keep), dtype=torch.float32, device=device)
    running = [[] for _ in range(beams)]
    running_scores = [0.] + [-1e9] * (beams - 1)
    seen, seen_next = ops.seen_bitmap(beams, vocab, device), ops.seen_bitmap(beams, vocab, device)
    finished = []
    improvable = True
    host = torch.empty(2 * keep + 2, dtype=torch.float64, pin_memory=True)
    out = {}
    for step in range(max_new_tokens):
        scores_t = torch.tensor(running_scores, dtype=torch.float32, device=device)
        out = ops.beam_step(logits.reshape(-1, vocab), scores_t, uniforms[step], seen_bits=seen,
                            temperature=temperature, top_p=top_p, top_k=TOP_K, keep=2,
                            repetition_penalty=REPETITION_PENALTY, num_picks=keep, out=out)
        # One device->host transfer for picks, picked scores, count and status.
        packed = torch.cat((out["picks"].double(), out["scores"].double(), out["n"].double(),
                            out["status"].double()))
        host.copy_(packed, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        vals = host.tolist()
        n, status = int(vals[2 * keep]), int(vals[2 * keep + 1])
        if status:
            _raise_status(status)
        picks = [int(v) for v in vals[:n]]
        picked = vals[keep:keep + n]  # float32 scores, exact as doubles (:236)
        parents, tokens = zip(*(divmod(pick, vocab) for pick in picks))
        candidates = [running[parent] + [token] for parent, token in zip(parents, tokens)]
        last = step + 1 == max_new_tokens
        hits = [last or _ends(candidate, stop_ids, eos_id) for candidate in candidates]
        if improvable and len(finished) < beams:
            finished += [(picked[j] / (step + 1) ** LENGTH_PENALTY, candidates[j])
                         for j in range(min(beams, len(picked))) if hits[j]]
            finished = sorted(finished, key=lambda item: item[0], reverse=True)[:beams]
        live = [score - 1e9 * hit for score, hit in zip(picked, hits)]
        order = sorted(range(len(picked)), key=live.__getitem__, reverse=True)[:beams]
        running_scores = [live[j] for j in order] + [-1e9] * (beams - len(order))
        order += [order[0]] * (beams - len(order))
        running = [candidates[j] for j in order]
        on_step(step + 1)
        worst = min(score for score, _ in finished) if len(finished) == beams else -1e9
        improvable = improvable and running_scores[0] / (step + 1) ** LENGTH_PENALTY > worst
        if not improvable or len(finished) == beams or all(hits):
            break
        if loop_guard and step % 16 == 15 and _repeating(running[0], device):
            return (finished[0][1] if finished else running[0]), 'repetition'
        selected = torch.tensor([parents[j] for j in order], dtype=torch.int64, device=device)
        next_tokens = torch.tensor([tokens[j] for j in order], dtype=torch.int64, device=device)
        ops.seen_reorder(seen, seen_next, selected, next_tokens, vocab)
        seen, seen_next = seen_next, seen
        decoding.reorder([parents[j] for j in order])
        logits = decoding.step(next_tokens)
    if not finished:
        return running[0], 'token_limit'
    best = finished[0][1]
    return best, ('token_limit' if len(best) == max_new_tokens and not _ends(best, stop_ids, eos_id) else 'stop')


def install(module) -> None:
    """Rebind the reference module's sampling functions to these (its own
    `generate_tokens`, runtime_shared.py:268-342, then runs the kernels)."""
    for name in ("_repeating", "_penalize", "_warp", "_sample", "_beam_sample"):
        setattr(module, name, globals()[name])
