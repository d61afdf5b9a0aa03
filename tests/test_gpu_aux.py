"""GPU parity of the drop-in's element-wise helpers against the reference's rules,
through the C ABI: the penalty alone (sv_penalize, runtime_shared.py:170-173) and
the beam step's seen-mask reorder (sv_seen_reorder, runtime_shared.py:258-259); and
the batched kernel's bounded wait running out (SV_ST_TIMEOUT) without losing the
context."""
import numpy as np
import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
DEV = "cuda"


def penalized_fp32(x, seen, rp=3.1):
    """seen ? (x < 0 ? x * 3.1f : x / 3.1f) : x in IEEE fp32, as torch's CPU kernels."""
    x = x.astype(np.float32)
    r = np.float32(rp)
    return np.where(seen, np.where(x < 0, x * r, x / r).astype(np.float32), x).astype(np.float32)


def packed_bits(seen):
    b = np.packbits(seen.astype(bool), axis=1, bitorder="little")
    b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int32)).to(DEV)


@pytest.mark.parametrize("form", ["mask8", "bits32"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("vocab", [49152, 49157, 1003])
def test_penalize_bit_exact(sv, form, dtype, vocab):
    g = np.random.default_rng(vocab)
    if vocab == 49152:
        d = bench.cfg1()
        x = np.repeat(d["logits"], 3, 0)
        x[1] *= -1
        x[2, ::7] = 0.0
    else:
        x = (3 * g.standard_normal((3, vocab))).astype(np.float32)
    seen = g.random((3, vocab)) < 0.3
    xd = torch.from_numpy(x).to(DEV).to(dtype)
    xf = xd.float().cpu().numpy()  # the values the kernel sees
    kw = {"seen": torch.from_numpy(seen).to(DEV)} if form == "mask8" else {"seen_bits": packed_bits(seen)}
    out = sv.penalize(xd, **kw).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), penalized_fp32(xf, seen).view(np.uint32))


def test_penalize_special_values(sv):
    x = np.array([[np.inf, -np.inf, np.nan, -0.0, 0.0, 1e-45, -1e-45, 3.4e38, -3.4e38]], np.float32)
    seen = np.ones_like(x, bool)
    out = sv.penalize(torch.from_numpy(x).to(DEV), seen=torch.from_numpy(seen).to(DEV)).cpu().numpy()
    ref = penalized_fp32(x, seen)
    np.testing.assert_array_equal(np.isnan(out), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_array_equal(out[ok].view(np.uint32), ref[ok].view(np.uint32))


@pytest.mark.parametrize("beams,vocab", [(2, 49152), (8, 49157), (5, 100)])
def test_seen_reorder_matches_reference_rule(sv, beams, vocab):
    """dst = seen[selected]; dst[arange(beams), next_tokens] = True (runtime_shared.py:258-259)."""
    g = np.random.default_rng(beams * vocab)
    words = (vocab + 31) // 32
    for trial in range(4):
        seen = g.random((beams, vocab)) < 0.05
        parents = g.integers(0, beams, beams)
        if trial == 0:
            parents[:] = 0  # every row continues beam 0
        tokens = g.integers(0, vocab, beams)
        src = packed_bits(seen)
        dst = torch.full_like(src, -1)
        sv.seen_reorder(src, dst, torch.from_numpy(parents).to(DEV), torch.from_numpy(tokens).to(DEV), vocab)
        ref = torch.from_numpy(seen)[torch.from_numpy(parents)]
        ref[torch.arange(beams), torch.from_numpy(tokens)] = True
        got = np.unpackbits(dst.cpu().numpy().view(np.uint8), axis=1, bitorder="little")
        np.testing.assert_array_equal(got[:, :vocab].astype(bool), ref.numpy())
        assert not got[:, vocab:words * 32].any()  # padding bits stay clear


def test_history_wait_timeout_reports_status_and_context_survives(sv):
    """The bounded wait on the history copy (SV_ST_TIMEOUT): the test hook makes the
    copy's barrier expect 16 bytes the copy never brings, so the wait runs out (after
    ~2 ms instead of ~1 s); every row reports status 5 and token -1, and the next,
    normal call on the same context gives the oracle's tokens."""
    import bench
    from oracle import oracle as O
    d = bench.cfg4(seed=5, rows=8, vocab=4096, hist_len=512)
    x = torch.from_numpy(d["logits"]).cuda()
    h = torch.from_numpy(d["history"]).cuda()
    u = torch.from_numpy(d["uniforms"]).cuda()
    for _ in range(2):
        o = sv.sample_step(x, u, history=h, path="stream", test_wait_timeout=True)
        torch.cuda.synchronize()
        assert o["status"].tolist() == [sv._lib.ST_TIMEOUT] * 8
        assert o["token"].tolist() == [-1] * 8
    o = sv.sample_step(x, u, history=h, path="stream")
    lengths = np.full(8, d["history"].shape[1], np.int32)
    want = O.sample(d["logits"], d["uniforms"], ids=d["history"], lengths=lengths, temperature=1.5, top_p=0.9)
    assert o["status"].tolist() == [0] * 8
    np.testing.assert_array_equal(o["token"].cpu().numpy(), want["token"])
