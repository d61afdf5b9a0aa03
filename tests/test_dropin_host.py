"""Host-side behaviour of the drop-in generate_tokens that needs no GPU: the
reference's argument validation (runtime_shared.py:277-300) raises ValueError
before any kernel runs (tests/test_generation.py:91-107 of the reference)."""
import pytest
import torch

from test_gpu_dropin import TinyTokenizer


class CpuDecoder:
    context, vocab = 40, 128

    def embed(self, ids):
        return torch.zeros((*ids.shape, 4))

    def prefill(self, embeddings, rows, capacity):  # never reached
        raise AssertionError("validation must fail before prefill")


@pytest.fixture
def rs(sv):
    import importlib
    return importlib.import_module("starvector_b200.runtime_shared")


@pytest.mark.parametrize("beams", [0, 9, 1.5, "2"])
def test_invalid_beam_count(rs, beams):
    with pytest.raises(ValueError, match="num_beams"):
        rs.generate_tokens(CpuDecoder(), TinyTokenizer(), torch.zeros(1, 8, 4), max_new_tokens=8, num_beams=beams)


def test_context_overflow(rs):
    with pytest.raises(ValueError, match="context size"):
        rs.generate_tokens(CpuDecoder(), TinyTokenizer(), torch.zeros(1, 39, 4), 4)


@pytest.mark.parametrize("temperature,top_p", [(0, 0.9), (-0.5, 0.9), (1, 0), (1, 1.1)])
def test_invalid_sampling_settings(rs, temperature, top_p):
    with pytest.raises(ValueError):
        rs.generate_tokens(CpuDecoder(), TinyTokenizer(), torch.zeros(1, 8, 4), max_new_tokens=8,
                           temperature=temperature, top_p=top_p)


def test_cpu_logits_are_rejected_not_sampled_on_cpu(sv):
    """No CPU fallback: CPU tensors raise instead of being sampled on the host."""
    with pytest.raises(RuntimeError, match="CUDA"):
        sv.sample_step(torch.zeros(1, 100), torch.zeros(1))


def test_constants_match_reference(rs):
    assert (rs.TOP_K, rs.REPETITION_PENALTY, rs.LENGTH_PENALTY, rs.LOOP_WINDOW, rs.LOOP_REPEATS) == \
        (50, 3.1, -1.0, 64, 3)
