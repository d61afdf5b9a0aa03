"""GPU parity of the beam KV-cache reorder (sv_kv_reorder) against the reference's
CachedDecoding.reorder (runtime_shared.py:388-394): rows whose parent changed take
the parent's keys and values over the first `length` slots, copied as torch's
advanced indexing copies them (sources read before rows are written); other rows
and slots past `length` are untouched.  Exact copies: compared bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference_reorder(keys, values, parents, length):
    """runtime_shared.py:388-394 on a copy."""
    k, v = keys.clone(), values.clone()
    rows = [row for row, parent in enumerate(parents) if parent != row]
    if rows:
        sources = [parents[row] for row in rows]
        k[:, rows, ..., :length, :] = k[:, sources, ..., :length, :]
        v[:, rows, ..., :length, :] = v[:, sources, ..., :length, :]
    return k, v


PARENTS = {2: [[0, 0], [1, 0], [1, 1], [0, 1]],
           8: [[0, 0, 0, 0, 0, 0, 0, 0], [1, 0, 3, 2, 5, 4, 7, 6], [0, 1, 2, 3, 4, 5, 6, 7], [7, 7, 1, 1, 0, 2, 6, 3]]}


@pytest.mark.parametrize("layout", ["mqa_1b", "gqa_8b"])
@pytest.mark.parametrize("beams", [2, 8])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_reorder_matches_reference(sv, layout, beams, dtype):
    g = torch.Generator(device=DEV).manual_seed(beams)
    if layout == "mqa_1b":   # GPTBigCode 1B: one key/value head
        shape = (6, beams, 300, 128)
    else:                    # StarCoder2 7B: grouped kv heads
        shape = (4, beams, 4, 300, 128)
    keys = torch.randn(shape, generator=g, device=DEV).to(dtype)
    values = torch.randn(shape, generator=g, device=DEV).to(dtype)
    for length in (1, 217, 300):
        for parents in PARENTS[beams]:
            ref_k, ref_v = reference_reorder(keys, values, parents, length)
            k, v = keys.clone(), values.clone()
            status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
            sv.ops.kv_reorder(k, v, torch.tensor(parents, dtype=torch.int64, device=DEV), length, out_status=status)
            torch.cuda.synchronize()
            assert status.item() == 0
            assert torch.equal(k.view(torch.uint8), ref_k.view(torch.uint8))  # bit for bit
            assert torch.equal(v.view(torch.uint8), ref_v.view(torch.uint8))


def test_invalid_parent_leaves_its_row(sv):
    keys = torch.randn((2, 3, 64, 64), device=DEV, dtype=torch.float16)
    values = torch.randn_like(keys)
    k, v = keys.clone(), values.clone()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    sv.ops.kv_reorder(k, v, torch.tensor([1, 7, 0], dtype=torch.int64, device=DEV), 64, out_status=status)
    torch.cuda.synchronize()
    assert status.item() == 1
    assert torch.equal(k[:, 1], keys[:, 1]) and torch.equal(k[:, 0], keys[:, 1]) and torch.equal(k[:, 2], keys[:, 0])


def test_keys_only_and_capture(sv):
    """values = None; and the call inside a CUDA graph (parents read on the device
    at replay time)."""
    keys = torch.randn((3, 4, 128, 64), device=DEV, dtype=torch.bfloat16)
    parents = torch.tensor([0, 1, 2, 3], dtype=torch.int64, device=DEV)
    work = keys.clone()
    sv.ops.kv_reorder(work, None, parents, 100)  # identity parents: nothing moves
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sv.ops.kv_reorder(work, None, parents, 100)
    parents.copy_(torch.tensor([3, 3, 0, 1], device=DEV))
    graph.replay()
    torch.cuda.synchronize()
    ref_k, _ = reference_reorder(keys, keys, [3, 3, 0, 1], 100)
    assert torch.equal(work, ref_k)
