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


def test_candidate_nodes_end_like_the_reference_lists(rs):
    """The beam replay holds candidates as linked nodes (token, parent node); its
    _ends on a node must equal the reference's _ends on the token list
    (runtime_shared.py:190-191) for every stop form: a list (matched), an empty
    list (never matches a non-empty candidate) and a tuple (a list slice never
    equals a tuple)."""
    import random
    rng = random.Random(7)
    for stop in ([3, 4], [3], [], (3, 4), [4, 3, 4]):
        for _ in range(300):
            seq = [rng.choice([3, 4, 5]) for _ in range(rng.randint(1, 7))]
            node = None
            for t in seq:
                node = (t, node)
            assert rs._node_tokens(node) == seq
            assert rs._node_tokens(node, 2) == seq[-2:]
            for eos in (5, None, 99):
                assert rs._node_ends(node, stop, eos) == rs._ends(seq, stop, eos), (seq, stop, eos)


def test_guard_table_sizes(sv):
    """The incremental loop guard's table: a power of two, at least twice the
    windows it will hold, all bits set (empty)."""
    for windows, want in ((1, 64), (32, 64), (33, 128), (4096, 8192), (4097, 16384)):
        t = sv.ops.guard_table(windows, "cpu")
        assert t.numel() == want and t.dtype == torch.int64 and bool((t == -1).all())


def test_device_reorder_detection(rs):
    """Which decoders the beam loop reorders from device parents: one that offers
    reorder_device; the reference's CachedDecoding (by class, with a CUDA cache of
    the beams' rows); anything else gets the reference's reorder(list)."""
    class WithHook:
        def reorder_device(self, parents):
            pass

    hook = WithHook()
    assert rs._device_reorder(hook, 2) == hook.reorder_device

    class CachedDecoding:  # the reference's class name, but a CPU cache: not on the device path
        def __init__(self):
            self.keys = torch.zeros((2, 2, 8, 16))
            self.values = torch.zeros_like(self.keys)
            self.length = 4

    assert rs._device_reorder(CachedDecoding(), 2) is None

    class Other:
        keys = values = None
        length = 0

    assert rs._device_reorder(Other(), 2) is None
