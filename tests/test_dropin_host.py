"""Host-side behaviour of the drop-in that needs no GPU: the binding into the
reference's module, the reference's constants, and no CPU fallback."""
import types

import pytest
import torch


@pytest.fixture
def rs(sv):
    import importlib
    return importlib.import_module("starvector_b200.runtime_shared")


def test_install_rebinds_the_sampling_functions(rs):
    """install() rebinds the names the reference's generate_tokens calls through
    its module globals (runtime_shared.py:316-319, :207, :254) and leaves the rest."""
    ref = types.ModuleType("runtime_shared")
    originals = {}
    for name in ("_repeating", "_penalize", "_warp", "_sample", "_beam_sample", "_ends", "generate_tokens"):
        originals[name] = lambda *a, **k: None
        setattr(ref, name, originals[name])
    rs.install(ref)
    for name in ("_repeating", "_penalize", "_warp", "_sample", "_beam_sample"):
        assert getattr(ref, name) is getattr(rs, name)
    assert ref._ends is originals["_ends"]
    assert ref.generate_tokens is originals["generate_tokens"]
    assert not hasattr(rs, "generate_tokens")


def test_cpu_logits_are_rejected_not_sampled_on_cpu(sv):
    """No CPU fallback: CPU tensors raise instead of being sampled on the host."""
    with pytest.raises(RuntimeError, match="CUDA"):
        sv.sample_step(torch.zeros(1, 100), torch.zeros(1))


def test_constants_match_reference(rs):
    assert (rs.TOP_K, rs.REPETITION_PENALTY, rs.LENGTH_PENALTY, rs.LOOP_WINDOW, rs.LOOP_REPEATS) == \
        (50, 3.1, -1.0, 64, 3)
