"""The reference's CPU sampling chain in torch: the timed CPU baseline (test
infrastructure only).

Only bench.py's CPU-baseline leg and its `--impl reference` arm run this module.
It is the timing baseline, not a checker (the C oracle in sv_oracle.c is the
checker): the reference (ComfyUI-StarVector-GGUF, a Python ComfyUI node) cannot
travel to the GPU box, so its chain is spelled here with the same torch calls in
the same order:
  * penalty (runtime_shared.py:170-173): torch.where over the cumulative bool
    `seen` mask;
  * temperature, top-k and top-p (:176-187): division, torch.topk threshold with
    ties, ascending torch.sort + softmax + cumsum for top-p, scatter back;
  * draw (:200-202): softmax, torch.multinomial(probs, 1), then `seen[token] = True`.
The rows of a step are batched into one call of each op (the reference's functions
take any leading shape), on every host thread torch is allowed to use.
"""
from __future__ import annotations

import time

import torch

TOP_K = 50
REPETITION_PENALTY = 3.1


def penalize(scores, seen, rp=REPETITION_PENALTY):
    """runtime_shared.py:170-173."""
    penalized = torch.where(scores < 0, scores * rp, scores / rp)
    return torch.where(seen, penalized, scores)


def warp(scores, temperature, top_p, keep, top_k=TOP_K):
    """runtime_shared.py:176-187."""
    if temperature != 1.0:
        scores = scores / temperature
    threshold = torch.topk(scores, max(top_k, keep))[0][..., -1:]
    scores = scores.masked_fill(scores < threshold, float("-inf"))
    if top_p < 1.0:
        ordered, order = torch.sort(scores, descending=False)
        remove = ordered.softmax(-1).cumsum(-1) <= 1 - top_p
        remove[..., -keep:] = False
        scores = scores.masked_fill(remove.scatter(-1, order, remove), float("-inf"))
    return scores


def seen_mask(history, vocab):
    """The reference's cumulative bool mask [rows, V] of each row's generated tokens."""
    h = torch.as_tensor(history, dtype=torch.int64)
    seen = torch.zeros((h.shape[0], vocab), dtype=torch.bool)
    seen.scatter_(1, h, True)
    return seen


def sample_step(logits, seen, temperature=1.5, top_p=0.9, generator=None):
    """One sample step for every row (runtime_shared.py:200-202): returns the tokens
    and sets their bits in `seen`."""
    scores = warp(penalize(logits, seen), temperature, top_p, 1)
    token = torch.multinomial(scores.softmax(-1), 1, generator=generator)
    seen.scatter_(1, token, True)
    return token[:, 0]


def rows_per_s(logits, seen, seconds=10.0, chunk=64, threads=None):
    """Rows/s of sample_step over chunks of `chunk` rows until `seconds` pass, on
    `threads` host threads (all when None); returns (rows/s, rows, seconds)."""
    old = torch.get_num_threads()
    if threads:
        torch.set_num_threads(threads)
    try:
        x = torch.as_tensor(logits)
        n = x.shape[0]
        g = torch.Generator().manual_seed(0)
        rows, i = 0, 0
        t0 = time.perf_counter()
        while True:
            s = slice(i, min(i + chunk, n))
            sample_step(x[s], seen[s], generator=g)
            rows += s.stop - s.start
            i = s.stop % n
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
    finally:
        torch.set_num_threads(old)
    return rows / dt, rows, dt
