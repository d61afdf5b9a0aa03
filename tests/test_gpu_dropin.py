"""The reference's generation-loop tests (tests/test_generation.py:52-122 of
ComfyUI-StarVector-GGUF), run against the drop-in's _sample / _beam_sample on CUDA.

The reference's generate_tokens (runtime_shared.py:268-342) stays the caller;
`generate` below makes the same calls it does (prompt embeddings appended to the
image prefix, max_new_tokens capped by the context, the seed set inside fork_rng,
:301-319).  The fake decoder makes one scripted token dominant (logit 200), so
outcomes do not depend on the draw rule: the same assertions as the reference's
must hold.  The decoder also checks that it is only ever fed valid token ids.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


class TinyTokenizer:
    eos_token_id = 99

    def encode(self, text):
        return {"<svg": [1, 2], "</svg>": [3, 4]}[text]

    def decode(self, ids):
        return "<svg" + "".join(f" {token}" for token in ids[2:])


class CudaScriptDecoder:
    """Every row's next-token logits put 200 on script[step] (then its last entry)."""

    def __init__(self, script, context=40, vocab=128, dtype=torch.float32):
        self.script, self.context, self.vocab, self.dtype = script, context, vocab, dtype
        self.calls = []

    def embed(self, ids):
        return torch.zeros((*ids.shape, 4), device=DEV)

    def prefill(self, embeddings, rows, capacity):
        self.calls.append(("prefill", embeddings.shape[1], rows, capacity))
        self.step_index = 0
        return self, self._logits(rows)

    def _logits(self, rows):
        logits = torch.zeros((rows, self.vocab), device=DEV, dtype=self.dtype)
        logits[:, self.script[min(self.step_index, len(self.script) - 1)]] = 200.
        return logits

    def step(self, tokens):
        ids = tokens.tolist()
        # An out-of-range id would be an embedding fault in a real decoder.
        assert all(0 <= t < self.vocab for t in ids), ids
        self.calls.append(("step", ids))
        self.step_index += 1
        return self._logits(tokens.shape[0])

    def reorder(self, parents):
        self.calls.append(("reorder", list(parents)))


@pytest.fixture
def rs(sv):
    import importlib
    return importlib.import_module("starvector_b200.runtime_shared")


def generate(rs, decoder, prefix, max_new_tokens=4096, num_beams=2, loop_guard=True, progress_callback=None,
             seed=0):
    """The drop-in's sampling loops called as the reference's generate_tokens calls
    them; returns (decoded text, stop reason)."""
    tok = TinyTokenizer()
    prompt_ids, stop_ids = tok.encode("<svg"), tok.encode("</svg>")
    max_new = min(int(max_new_tokens), decoder.context - prefix.shape[1] - len(prompt_ids))
    embeddings = torch.cat((prefix, decoder.embed(torch.tensor([prompt_ids], device=DEV))), dim=1)
    on_step = progress_callback if progress_callback is not None else (lambda step: None)
    with torch.inference_mode(), torch.random.fork_rng(devices=[torch.cuda.current_device()]):
        torch.manual_seed(seed)
        if num_beams == 1:
            generated, reason = rs._sample(decoder, embeddings, max_new, 1.5, 0.9, stop_ids, tok.eos_token_id,
                                           loop_guard, on_step)
        else:
            generated, reason = rs._beam_sample(decoder, embeddings, max_new, 1.5, 0.9, num_beams, stop_ids,
                                                tok.eos_token_id, loop_guard, on_step)
    return tok.decode(prompt_ids + generated), reason


@pytest.mark.parametrize("beams", [1, 2, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_generates_until_svg_end(rs, beams, dtype):
    decoder = CudaScriptDecoder([7, 8, 3, 4, 9], dtype=dtype)
    svg, reason = generate(rs, decoder, torch.zeros(1, 8, 4, device=DEV), max_new_tokens=16, num_beams=beams)
    assert svg == "<svg 7 8 3 4"
    assert reason == "stop"
    assert decoder.calls[0] == ("prefill", 10, beams, 26)


def test_generation_emits_incremental_progress(rs):
    events = []
    generate(rs, CudaScriptDecoder([7, 3, 4]), torch.zeros(1, 8, 4, device=DEV), max_new_tokens=8, num_beams=1,
             progress_callback=events.append)
    assert events == [1, 2, 3]


@pytest.mark.parametrize("beams", [1, 2])
def test_token_limit(rs, beams):
    decoder = CudaScriptDecoder([7])
    svg, reason = generate(rs, decoder, torch.zeros(1, 34, 4, device=DEV), max_new_tokens=4096, num_beams=beams)
    assert svg == "<svg 7 7 7 7"
    assert reason == "token_limit"
    assert decoder.calls[0] == ("prefill", 36, beams, 40)


@pytest.mark.parametrize("beams", [1, 2])
def test_loop_guard_stops_repeated_output(rs, beams):
    script = list(range(5, 69)) * 20
    svg, reason = generate(rs, CudaScriptDecoder(script, context=2000), torch.zeros(1, 8, 4, device=DEV),
                           max_new_tokens=1000, num_beams=beams)
    generated = len(svg.split()) - 1
    assert 64 * 3 <= generated < 64 * 3 + 16
    assert reason == "repetition"
    svg, reason = generate(rs, CudaScriptDecoder(script, context=2000), torch.zeros(1, 8, 4, device=DEV),
                           max_new_tokens=1000, num_beams=beams, loop_guard=False)
    assert len(svg.split()) - 1 == 1000
    assert reason == "token_limit"


def test_processors_match_transformers(rs):
    from transformers import (RepetitionPenaltyLogitsProcessor, TemperatureLogitsWarper, TopKLogitsWarper,
                              TopPLogitsWarper)
    torch.manual_seed(0)
    scores = torch.randn(3, 200) * 4
    history = torch.tensor([[5, 9, 9], [0, 1, 2], [7, 150, 199]])
    seen = torch.zeros_like(scores, dtype=torch.bool).scatter(1, history, True)
    for keep in (1, 2):
        expected = RepetitionPenaltyLogitsProcessor(rs.REPETITION_PENALTY)(history, scores.clone())
        for processor in (TemperatureLogitsWarper(1.5), TopKLogitsWarper(rs.TOP_K, min_tokens_to_keep=keep),
                          TopPLogitsWarper(0.9, min_tokens_to_keep=keep)):
            expected = processor(history, expected)
        actual = rs._warp(rs._penalize(scores.to(DEV), seen.to(DEV)), 1.5, 0.9, keep).cpu()
        assert torch.equal(torch.isinf(actual), torch.isinf(expected))
        assert torch.allclose(actual[torch.isfinite(actual)], expected[torch.isfinite(expected)])


def test_repeating_matches_reference_rule(rs):
    script = list(range(5, 69)) * 4
    assert not rs._repeating(script[:191])
    assert rs._repeating(script[:192])
    assert not rs._repeating(list(range(300)))


def test_stop_inside_a_read_block(rs):
    """The host reads sampled tokens once per 16 steps: an end at step 21 still
    stops there, with the progress callback called once per step up to it."""
    events = []
    script = [7] * 19 + [3, 4] + [8] * 20
    svg, reason = generate(rs, CudaScriptDecoder(script), torch.zeros(1, 8, 4, device=DEV), max_new_tokens=30,
                           num_beams=1, progress_callback=events.append)
    assert svg == "<svg" + " 7" * 19 + " 3 4"
    assert reason == "stop"
    assert events == list(range(1, 22))


class NanAtStepDecoder(CudaScriptDecoder):
    def _logits(self, rows):
        logits = super()._logits(rows)
        if self.step_index == 9:
            logits[:, 5] = float("nan")
        return logits


def test_error_status_inside_a_read_block(rs):
    """A step whose logits hold a NaN raises the reference's error even though the
    host reads the steps' statuses only once per 16 steps; the decode steps issued
    after the failed one inside the block are fed valid ids (the decoder asserts it)."""
    events = []
    decoder = NanAtStepDecoder([7])
    with pytest.raises(RuntimeError, match="probability tensor contains"):
        generate(rs, decoder, torch.zeros(1, 8, 4, device=DEV), max_new_tokens=30, num_beams=1,
                 progress_callback=events.append)
    assert events == list(range(1, 10))
    fed = [c[1][0] for c in decoder.calls if c[0] == "step"]
    assert fed == [7] * 9 + [0] + [7] * 5  # the failed step 9 is fed as token 0


class CachedDecoding:
    """A scripted decoder with the reference's CachedDecoding cache protocol
    (runtime_shared.py:345-394): keys / values [layers, rows, capacity, head_dim],
    `length`, `reorder(parents)` by torch indexing.  The drop-in recognises the
    class and reorders the cache on the device from device parents.  Each step
    writes the fed token into its cache slot, so the final cache records every
    row's ancestry; logits are seeded per step (random, so beams branch); fed ids
    are checked on the device (no host sync)."""

    def __init__(self, vocab=64, context=200, rows=2, seed=0, never=()):
        self.vocab, self.context, self.seed = vocab, context, seed
        self.never = torch.tensor(list(never), dtype=torch.int64, device=DEV)
        self.bad = torch.zeros((), dtype=torch.bool, device=DEV)

    def embed(self, ids):
        return torch.zeros((*ids.shape, 4), device=DEV)

    def prefill(self, embeddings, rows, capacity):
        self.rows, self.length, self.index = rows, embeddings.shape[1], 0
        self.keys = torch.zeros((2, rows, capacity, 8), device=DEV)
        self.values = torch.zeros_like(self.keys)
        # Every step's logits made up front, so a step launches no random kernels.
        g = torch.Generator(device=DEV).manual_seed(self.seed)
        self.table = torch.randn((capacity - self.length + 1, rows, self.vocab), generator=g, device=DEV) * 3
        self.table[:, :, self.never] = -60.  # ids that are never drawn
        return self, self._logits()

    def _logits(self):
        return self.table[self.index]

    def step(self, tokens):
        self.bad |= ((tokens < 0) | (tokens >= self.vocab)).any()
        self.keys[:, :, self.length, 0] = tokens.float()
        self.values[:, :, self.length, 1] = tokens.float() + 0.5
        self.length += 1
        self.index += 1
        return self._logits()

    def reorder(self, parents):
        rows = [row for row, parent in enumerate(parents) if parent != row]
        if rows:
            sources = [parents[row] for row in rows]
            self.keys[:, rows, ..., :self.length, :] = self.keys[:, sources, ..., :self.length, :]
            self.values[:, rows, ..., :self.length, :] = self.values[:, sources, ..., :self.length, :]


class HostDecoding(CachedDecoding):
    """The same decoder under another name: the drop-in reorders it from host lists,
    one step at a time."""


@pytest.mark.parametrize("beams", [2, 3, 8])
@pytest.mark.parametrize("loop_guard", [True, False])
def test_device_decision_equals_host_path(rs, beams, loop_guard):
    """The 16-step device-driven loop and the per-step host-driven loop give the same
    tokens, reason, callbacks and final cache (stop ids and eos drawn by chance from
    64 tokens, so generations end at varied steps)."""
    for seed in range(6):
        runs = []
        for cls in (CachedDecoding, HostDecoding):
            decoder, events = cls(seed=seed), []
            svg, reason = generate(rs, decoder, torch.zeros(1, 8, 4, device=DEV), max_new_tokens=150,
                                   num_beams=beams, loop_guard=loop_guard, progress_callback=events.append, seed=seed)
            assert not bool(decoder.bad)
            runs.append((svg, reason, events, decoder.keys[:, :, :decoder.length].clone(),
                         decoder.values[:, :, :decoder.length].clone()))
        (s1, r1, e1, k1, v1), (s2, r2, e2, k2, v2) = runs
        assert (s1, r1, e1) == (s2, r2, e2)
        # The device loop may run up to 15 steps past the end: compare the slots
        # both wrote.
        n = min(k1.shape[2], k2.shape[2])
        assert torch.equal(k1[:, :, :n], k2[:, :, :n]) and torch.equal(v1[:, :, :n], v2[:, :, :n])


def test_beam_loop_syncs_once_per_block(rs):
    """With a decoder reordered on the device, the beam loop's host synchronisations
    are one per 16 steps (plus setup), not one per token."""
    import traceback
    import warnings
    decoder = CachedDecoding(vocab=4096, context=200, seed=3, never=[4000, 4001, 4002])
    steps = 96
    sites = []

    def record(message, category, filename, lineno, file=None, line=None):
        if "called a synchronizing" in str(message):
            frames = [f for f in traceback.extract_stack()[:-1] if not f.filename.endswith("warnings.py")]
            sites.append(" < ".join(f"{f.filename.rsplit('/', 1)[-1]}:{f.lineno}" for f in frames[-3:][::-1]))

    torch.cuda.synchronize()
    with warnings.catch_warnings():
        warnings.simplefilter("always")
        warnings.showwarning = record
        torch.cuda.set_sync_debug_mode("warn")
        try:
            embeddings = torch.zeros(1, 10, 4, device=DEV)
            with torch.inference_mode():
                generated, reason = rs._beam_sample(decoder, embeddings, steps, 1.5, 0.9, 2, [4000, 4001], 4002,
                                                    False, lambda step: None)
        finally:
            torch.cuda.set_sync_debug_mode("default")
    assert reason == "token_limit" and len(generated) == steps
    assert steps // 16 <= len(sites) <= steps // 16 + 3, sorted(set(sites))
