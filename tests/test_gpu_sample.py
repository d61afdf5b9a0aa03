"""GPU parity of the fused sample-mode kernel against the CPU oracle (bit-exact),
through the C ABI (ops.sample_step -> sv_sample_step).

Every comparison is exact: token, kept count, kept ids, probabilities, warped
scores and dense outputs, because the kernel and the oracle implement the same
arithmetic (IEEE penalty/temperature, sv_exp, exact fixed-point sums).  The
oracle is pinned to the reference by tests/test_oracle_golden.py.
"""
import numpy as np
import pytest
import torch

import bench
from _golden import explain_mismatch, load, names, row_sparse, tempered
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t.to(dtype) if dtype is not None else t


PATHS = ["cluster", "stream"]


def run_both(sv, x, u, *, ids=None, seen=None, form="ids32", T=1.5, p=0.9, keep=1, top_k=50, cap=None,
             dtype=torch.float32, dense=True, force=False, path=None):
    R, Vv = x.shape
    cap = Vv if cap is None else cap
    xd = to_dev(x).to(dtype)
    xf = xd.float().cpu().numpy()  # the values the kernel sees
    kw = {}
    seen_np = seen
    if ids is not None:
        seen_np = O.seen_from_ids(ids, np.full(len(ids), ids.shape[1]), Vv)
        if form == "ids32":
            kw["history"] = to_dev(ids.astype(np.int32))
        elif form == "ids64":
            kw["history"] = to_dev(ids.astype(np.int64))
    if seen_np is not None and "history" not in kw:
        if form == "bits32":
            bits = np.packbits(seen_np.astype(bool), axis=1, bitorder="little")
            pad = (-bits.shape[1]) % 4
            bits = np.pad(bits, ((0, 0), (0, pad))).view(np.int32)
            kw["seen_bits"] = to_dev(bits)
        else:
            kw["seen"] = to_dev(seen_np.astype(bool))
    out = sv.sample_step(xd, to_dev(u), temperature=T, top_p=p, top_k=top_k, keep=keep, out_capacity=cap,
                         dense="probs" if dense else None, force_general=force, path=path, **kw)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in out.items()}
    ref = O.sample(xf, u, seen=seen_np, temperature=T, top_p=p, top_k=top_k, keep=keep, cap=cap, dense=dense)
    return got, ref


def assert_same(got, ref, dense=True):
    np.testing.assert_array_equal(got["status"], ref["status"])
    np.testing.assert_array_equal(got["token"], ref["token"])
    np.testing.assert_array_equal(got["count"], ref["count"])
    cap = got["idx"].shape[1]
    for r in range(len(got["token"])):
        n = min(int(ref["count"][r]), cap)
        np.testing.assert_array_equal(got["idx"][r, :n], ref["idx"][r, :n])
        np.testing.assert_array_equal(got["prob"][r, :n], ref["prob"][r, :n])
    if dense:
        np.testing.assert_array_equal(got["dense"], ref["probs"])


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("force", [False, True], ids=["fast", "general"])
@pytest.mark.parametrize("name", names("proc"))
def test_golden_cases(sv, name, force, path):
    d = load(name)
    x, seen = d["logits"], d["seen"]
    R = x.shape[0]
    T, p, keep = float(d["temperature"]), float(d["top_p"]), int(d["keep"])
    u = np.random.default_rng(7).random(R).astype(np.float32)
    got, ref = run_both(sv, x, u, seen=seen, form="mask8", T=T, p=p, keep=keep, force=force, path=path)
    assert_same(got, ref)
    # And against the reference's own output (golden): kept sets, bit-exact scores.
    out = sv.sample_step(to_dev(x), to_dev(u), seen=to_dev(seen), temperature=T, top_p=p, keep=keep,
                         dense="scores", force_general=force, path=path)
    dense = out["dense"].cpu().numpy()
    for r in range(R):
        gi, gv = row_sparse(d, r)
        oi = np.nonzero(np.isfinite(dense[r]))[0]
        assert explain_mismatch(tempered(x[r], seen[r], T), oi, gi, p, keep) is None
        common = np.intersect1d(oi, gi)
        np.testing.assert_array_equal(dense[r][common], gv[np.isin(gi, common)])


@pytest.mark.parametrize("form", ["ids32", "ids64", "mask8", "bits32", "none"])
@pytest.mark.parametrize("path", PATHS)
def test_history_forms(sv, form, path):
    g = np.random.default_rng(11)
    R, Vv = 6, 5000
    x = (2 * g.standard_normal((R, Vv))).astype(np.float32)
    ids = g.integers(0, Vv, (R, 700))
    u = g.random(R).astype(np.float32)
    if form == "none":
        got, ref = run_both(sv, x, u, form="none", path=path)
    else:
        got, ref = run_both(sv, x, u, ids=ids, form=form, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("vocab", [128, 1000, 4099, 49152, 49157])
@pytest.mark.parametrize("path", PATHS)
def test_dtypes_and_ragged_vocab(sv, dtype, vocab, path):
    g = np.random.default_rng(vocab)
    R = 3
    x = (2.5 * g.standard_normal((R, vocab))).astype(np.float32)
    ids = g.integers(0, vocab, (R, min(vocab, 300)))
    u = g.random(R).astype(np.float32)
    got, ref = run_both(sv, x, u, ids=ids, dtype=dtype, cap=128, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("T,p,keep", [(0.5, 0.9, 1), (1.0, 1.0, 1), (1.5, 0.5, 2), (3.0, 0.99, 1), (1.5, 0.9, 5),
                                      (0.05, 0.9, 1)])
@pytest.mark.parametrize("path", PATHS)
def test_temperature_top_p_keep(sv, T, p, keep, path):
    g = np.random.default_rng(int(T * 100) + keep)
    x = (2 * g.standard_normal((8, 8192))).astype(np.float32)
    ids = g.integers(0, 8192, (8, 500))
    u = g.random(8).astype(np.float32)
    got, ref = run_both(sv, x, u, ids=ids, T=T, p=p, keep=keep, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("top_k", [1, 7, 64, 128])
@pytest.mark.parametrize("path", PATHS)
def test_top_k_range(sv, top_k, path):
    g = np.random.default_rng(top_k)
    x = (2 * g.standard_normal((4, 20000))).astype(np.float32)
    u = g.random(4).astype(np.float32)
    got, ref = run_both(sv, x, u, ids=g.integers(0, 20000, (4, 100)), top_k=top_k, cap=256, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_ties_fp16_and_forced_general(sv, path):
    g = np.random.default_rng(5)
    x = np.round((3 * g.standard_normal((16, 49152))).astype(np.float16).astype(np.float32) * 2) / 2
    ids = g.integers(0, 49152, (16, 1000))
    u = g.random(16).astype(np.float32)
    for force in (False, True):
        got, ref = run_both(sv, x.astype(np.float32), u, ids=ids, dtype=torch.float16, force=force, cap=512, path=path)
        assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_huge_tie_group_takes_general_path(sv, path):
    """All-equal logits: top-k keeps every token (ties), top-p removes the lowest
    indices of the tie group; the candidate buffer overflows."""
    g = np.random.default_rng(6)
    x = np.zeros((3, 49152), np.float32)
    x[1, 17] = 3.0
    x[2, :100] = 1.0
    u = np.array([0.0, 0.5, 0.999999], np.float32)
    got, ref = run_both(sv, x, u, ids=g.integers(0, 49152, (3, 50)), cap=64, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_special_values(sv, path):
    g = np.random.default_rng(8)
    x = (2 * g.standard_normal((6, 3000))).astype(np.float32)
    x[0, 5] = np.nan
    x[1, 9] = np.inf
    x[2, :] = -np.inf
    x[3, g.choice(3000, 2990, replace=False)] = -np.inf  # 10 finite < top_k
    x[4, :] = -np.inf
    x[4, 123] = 1.0                                       # a single finite logit
    x[5, :] = 0.0                                         # exact zeros
    x[5, 7] = -0.0
    u = g.random(6).astype(np.float32)
    got, ref = run_both(sv, x, u, ids=g.integers(0, 3000, (6, 40)), path=path)
    np.testing.assert_array_equal(got["status"], [1, 2, 3, 0, 0, 0])
    assert_same(got, ref)


@pytest.mark.parametrize("force", [False, True])
@pytest.mark.parametrize("path", PATHS)
def test_error_precedence_and_temperature_overflow(sv, path, force):
    """A NaN anywhere in the row wins over a +inf before it; a finite score that the
    temperature (T < 1) takes to +inf is a +inf score, unless the penalty lowers it."""
    g = np.random.default_rng(10)
    x = (2 * g.standard_normal((5, 3000))).astype(np.float32)
    x[0, 9] = np.inf
    x[0, 2000] = np.nan
    x[1, 100] = 3.0e38   # / 0.5 overflows
    x[2, 100] = 3.0e38   # seen: / 3.1 first, then / 0.5 stays finite
    x[3, 7] = -3.0e38    # seen: * 3.1 gives -inf
    ids = g.integers(0, 3000, (5, 40))
    ids[:, 0] = [1, 2, 100, 7, 3]
    got, ref = run_both(sv, x, g.random(5).astype(np.float32), ids=ids, T=0.5, force=force, path=path)
    np.testing.assert_array_equal(got["status"], [1, 2, 0, 0, 0])
    assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_ascending_rows_and_dense_histories(sv, path):
    """Rows whose scores rise along the vocabulary (every chunk beats the bound
    so far: the streaming kernel's unit list overflows and the row is read again)
    and histories covering a quarter of the vocabulary."""
    g = np.random.default_rng(12)
    V = 49152
    x = (2 * g.standard_normal((8, V))).astype(np.float32)
    x[:4] += np.linspace(0.0, 12.0, V, dtype=np.float32)
    ids = g.integers(0, V, (8, 16384))
    got, ref = run_both(sv, x, g.random(8).astype(np.float32), ids=ids, cap=128, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_history_out_of_range_is_reported(sv, path):
    x = torch.zeros((2, 1000), device=DEV)
    hist = torch.tensor([[1, 2, 3], [4, 1000, 5]], dtype=torch.int32, device=DEV)
    out = sv.sample_step(x, torch.zeros(2, device=DEV), history=hist, path=path)
    assert out["status"].tolist() == [0, 4]
    assert out["token"].tolist()[1] == -1


@pytest.mark.parametrize("path", PATHS)
def test_broadcast_row_and_misaligned_base(sv, path):
    """Stride-0 rows (the prefill's expand, runtime_1b.py:82) and rows that start
    off the 16-byte grid (an offset view)."""
    g = np.random.default_rng(9)
    base = to_dev((2 * g.standard_normal(49157 * 3 + 3)).astype(np.float32))
    x = base[1:1 + 49157].reshape(1, -1).expand(4, -1)
    assert x.stride(0) == 0
    seen = torch.zeros((4, 49157), dtype=torch.bool, device=DEV)
    seen[1, :500] = True
    u = to_dev(g.random(4).astype(np.float32))
    out = sv.sample_step(x, u, seen=seen, out_capacity=64, path=path)
    xn = np.repeat(x[:1].cpu().numpy(), 4, 0)
    ref = O.sample(xn, u.cpu().numpy(), seen=seen.cpu().numpy(), cap=64)
    np.testing.assert_array_equal(out["token"].cpu().numpy(), ref["token"])
    np.testing.assert_array_equal(out["prob"].cpu().numpy(), ref["prob"])
    x2 = base[3:3 + 3 * 49151].reshape(3, 49151)
    xh = x2.half()[:, 1:]
    out = sv.sample_step(xh, u[:3], out_capacity=64, path=path)
    ref = O.sample(xh.float().cpu().numpy(), u[:3].cpu().numpy(), cap=64)
    np.testing.assert_array_equal(out["token"].cpu().numpy(), ref["token"])
    np.testing.assert_array_equal(out["prob"].cpu().numpy(), ref["prob"])


@pytest.mark.parametrize("path", PATHS)
def test_seen_update_in_kernel(sv, path):
    g = np.random.default_rng(10)
    x = to_dev((2 * g.standard_normal((5, 3000))).astype(np.float32))
    bits = sv.seen_bitmap(5, 3000, DEV)
    out = sv.sample_step(x, to_dev(g.random(5).astype(np.float32)), seen_bits=bits, update_seen_bits=bits,
                         path=path)
    tok = out["token"].cpu().numpy()
    b = bits.cpu().numpy().view(np.uint32)
    for r in range(5):
        set_bits = [w * 32 + i for w in range(b.shape[1]) for i in range(32) if (b[r, w] >> i) & 1]
        assert set_bits == [tok[r]]


@pytest.mark.parametrize("path", PATHS)
def test_uniform_edges_select_first_and_last(sv, path):
    g = np.random.default_rng(12)
    x = (2 * g.standard_normal((2, 4000))).astype(np.float32)
    u = np.array([0.0, np.nextafter(np.float32(1), np.float32(0))], np.float32)
    got, ref = run_both(sv, x, u, cap=100, path=path)
    assert_same(got, ref)
    n = got["count"]
    assert got["token"][0] == got["idx"][0, 0]
    assert got["token"][1] == got["idx"][1, n[1] - 1]


@pytest.mark.parametrize("path", PATHS)
def test_cfg1_full_size(sv, path):
    d = bench.cfg1()
    got, ref = run_both(sv, d["logits"], d["uniforms"], ids=d["history"], cap=256, path=path)
    assert_same(got, ref)


@pytest.mark.parametrize("path", PATHS)
def test_cfg4_full_size_against_oracle(sv, path):
    """Config 4 at its full size: 1024 rows x 49152, Zipf histories; every row
    bit-exact against the oracle, plus size-independent properties."""
    d = bench.cfg4()
    x, h, u = d["logits"], d["history"], d["uniforms"]
    out = sv.sample_step(to_dev(x), to_dev(u), history=to_dev(h), out_capacity=128, path=path)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in out.items()}
    ref = O.sample(x, u, ids=h, cap=128)
    assert_same(got, ref, dense=False)
    # Properties: the token is kept, probabilities sum to 1, ids ascending.
    for r in range(0, 1024, 37):
        n = got["count"][r]
        assert got["token"][r] in got["idx"][r, :n]
        assert abs(got["prob"][r, :n].astype(np.float64).sum() - 1) < 1e-5
        assert np.all(np.diff(got["idx"][r, :n]) > 0)


@pytest.mark.parametrize("vocab,dtype,dense,per_sm", [(5000, torch.float32, True, 7.05), (49152, torch.float16, False, 3.1),
                                                      (12345, torch.bfloat16, True, 0.7), (49157, torch.float32, False, 6.2)])
def test_stream_row_counts(sv, vocab, dtype, dense, per_sm):
    """The batched kernel at row counts that pick each of its CTA sizes (128, 256
    and 512 threads per row) and at more rows than fit the GPU at once; random
    settings, bit-exact against the oracle."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rows = int(per_sm * sms) + 3
    g = np.random.default_rng(vocab)
    x = (2 * g.standard_normal((rows, vocab))).astype(np.float32)
    x[::5, g.choice(vocab, 12, replace=False)] += 9.0
    u = g.random(rows).astype(np.float32)
    ids = g.integers(0, vocab, (rows, 300))
    got, ref = run_both(sv, x, u, ids=ids, T=1.3, p=0.85, dtype=dtype, dense=dense, cap=96, path="stream")
    assert_same(got, ref, dense=dense)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shift", [1, 3, 7, 13])
def test_stream_row_offsets(sv, dtype, shift):
    """Rows that start at every kind of offset from the 32-byte grid (a view into
    a larger buffer with an odd row stride), so the first and last units of each
    row are partial; bit-exact against the oracle."""
    g = np.random.default_rng(100 + shift)
    rows, V, stride = 70, 7001, 7001 + shift
    buf = (2 * g.standard_normal(rows * stride + 64)).astype(np.float32)
    full = to_dev(buf).to(dtype)
    x = full[shift:shift + rows * stride].reshape(rows, stride)[:, :V]
    ids = g.integers(0, V, (rows, 200))
    u = to_dev(g.random(rows).astype(np.float32))
    out = sv.sample_step(x, u, history=to_dev(ids.astype(np.int32)), out_capacity=64, path="stream")
    torch.cuda.synchronize()
    xf = x.float().cpu().numpy()
    ref = O.sample(xf, u.cpu().numpy(), ids=ids, cap=64)
    got = {k: v.cpu().numpy() for k, v in out.items()}
    assert_same(got, ref, dense=False)
