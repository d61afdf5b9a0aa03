"""The reference's generation-loop tests (tests/test_generation.py:52-122 of
ComfyUI-StarVector-GGUF), run against the drop-in runtime_shared on CUDA.

The fake decoder makes one scripted token dominant (logit 200), so outcomes do
not depend on the draw rule: the same assertions as the reference's must hold.
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
        self.calls.append(("step", tokens.tolist()))
        self.step_index += 1
        return self._logits(tokens.shape[0])

    def reorder(self, parents):
        self.calls.append(("reorder", list(parents)))


@pytest.fixture
def rs(sv):
    import importlib
    return importlib.import_module("starvector_b200.runtime_shared")


@pytest.mark.parametrize("beams", [1, 2, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_generates_until_svg_end(rs, beams, dtype):
    decoder = CudaScriptDecoder([7, 8, 3, 4, 9], dtype=dtype)
    cpu_before, cuda_before = torch.get_rng_state(), torch.cuda.get_rng_state()
    svg = rs.generate_tokens(decoder, TinyTokenizer(), torch.zeros(1, 8, 4, device=DEV), max_new_tokens=16,
                             num_beams=beams)
    assert svg == "<svg 7 8 3 4"
    assert decoder.calls[0] == ("prefill", 10, beams, 26)
    assert torch.equal(torch.get_rng_state(), cpu_before)
    assert torch.equal(torch.cuda.get_rng_state(), cuda_before)


def test_generation_emits_incremental_progress(rs):
    events = []
    rs.generate_tokens(CudaScriptDecoder([7, 3, 4]), TinyTokenizer(), torch.zeros(1, 8, 4, device=DEV),
                       max_new_tokens=8, num_beams=1, progress_callback=events.append)
    assert events == [1, 2, 3]


def test_context_cap(rs, caplog):
    decoder = CudaScriptDecoder([7])
    with caplog.at_level("INFO", logger=rs.__name__):
        svg = rs.generate_tokens(decoder, TinyTokenizer(), torch.zeros(1, 34, 4, device=DEV), max_new_tokens=4096,
                                 num_beams=1)
    assert "requested max_new_tokens=4096, effective max_new_tokens=4" in caplog.text
    assert svg == "<svg 7 7 7 7"
    assert decoder.calls[0] == ("prefill", 36, 1, 40)


@pytest.mark.parametrize("beams", [1, 2])
def test_loop_guard_stops_repeated_output(rs, beams, caplog):
    script = list(range(5, 69)) * 20
    with caplog.at_level("WARNING", logger=rs.__name__):
        svg = rs.generate_tokens(CudaScriptDecoder(script, context=2000), TinyTokenizer(),
                                 torch.zeros(1, 8, 4, device=DEV), max_new_tokens=1000, num_beams=beams)
    generated = len(svg.split()) - 1
    assert 64 * 3 <= generated < 64 * 3 + 16
    assert "loop guard" in caplog.text
    svg = rs.generate_tokens(CudaScriptDecoder(script, context=2000), TinyTokenizer(),
                             torch.zeros(1, 8, 4, device=DEV), max_new_tokens=1000, num_beams=beams, loop_guard=False)
    assert len(svg.split()) - 1 == 1000


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
    svg = rs.generate_tokens(CudaScriptDecoder(script), TinyTokenizer(), torch.zeros(1, 8, 4, device=DEV),
                             max_new_tokens=30, num_beams=1, progress_callback=events.append)
    assert svg == "<svg" + " 7" * 19 + " 3 4"
    assert events == list(range(1, 22))


class NanAtStepDecoder(CudaScriptDecoder):
    def _logits(self, rows):
        logits = super()._logits(rows)
        if self.step_index == 9:
            logits[:, 5] = float("nan")
        return logits


def test_error_status_inside_a_read_block(rs):
    """A step whose logits hold a NaN raises the reference's error even though the
    host reads the steps' statuses only once per 16 steps."""
    events = []
    with pytest.raises(RuntimeError, match="probability tensor contains"):
        rs.generate_tokens(NanAtStepDecoder([7]), TinyTokenizer(), torch.zeros(1, 8, 4, device=DEV),
                           max_new_tokens=30, num_beams=1, progress_callback=events.append)
    assert events == list(range(1, 10))
