"""The C-ABI library without a GPU: it loads, exports every function that
include/*.h declares, and rejects invalid arguments with the documented codes
before touching the device (no kernel launch, no CUDA call)."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(sv_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("sv_sample_step", "sv_beam_step", "sv_beam_workspace_bytes", "sv_loop_guard", "sv_penalize",
              "sv_seen_update", "sv_seen_reorder", "sv_error_string", "sv_abi_version"):
        assert n in names


def test_library_exports_every_declared_symbol(sv):
    lib = sv._lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", sv._lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(sv_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None


def test_abi_version_and_error_strings(sv):
    lib = sv._lib.lib()
    assert lib.sv_abi_version() == 1
    assert sv._lib.error_string(-4).startswith("temperature")
    assert sv._lib.error_string(1) == "NaN logit in row"


def test_workspace_size(sv):
    lib = sv._lib.lib()
    assert lib.sv_beam_workspace_bytes(2, 49152) > 2 * 49152 * 16
    assert lib.sv_beam_workspace_bytes(0, 10) == 0


def _sample(lib, **kw):
    args = dict(logits=8, dtype=0, rows=1, vocab=100, stride=100, hist=None, hkind=0, hstride=0, hlen=None, hcols=0,
                u=8, T=1.5, p=0.9, k=50, keep=1, rp=3.1, tok=8, cnt=None, idx=None, prob=None, score=None, cap=0,
                dense=None, dmode=0, dstride=0, st=None, bits=None, bstride=0, flags=0, stream=None)
    args.update(kw)
    return lib.sv_sample_step(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(logits=None), -1), (dict(dtype=7), -2), (dict(rows=0), -3), (dict(vocab=600000), -3),
    (dict(stride=50), -3), (dict(T=0.0), -4), (dict(T=-1.0), -4), (dict(p=0.0), -4), (dict(p=1.1), -4),
    (dict(k=0), -4), (dict(k=129), -4), (dict(keep=0), -4), (dict(vocab=40, stride=40), -4),
    (dict(logits=2), -5), (dict(u=None), -1), (dict(tok=None), -1), (dict(dmode=1), -1), (dict(hkind=9), -2),
    (dict(hkind=1, hist=None), -1), (dict(rp=0.0), -4),
])
def test_sample_step_rejects_invalid_arguments(sv, kw, code):
    assert _sample(sv._lib.lib(), **kw) == code


def test_beam_step_rejects_bad_workspace_and_counts(sv):
    lib = sv._lib.lib()
    base = [8, 0, 2, 100, 100, None, 0, 0, None, 0, 8, 8, 4, 1.5, 0.9, 50, 2, 3.1, 8, 8, 8, 8,
            None, None, None, None, 0, None, 0, 16, 0, 0, None]
    a = list(base)
    a[29] = 16
    a[30] = 10  # workspace too small
    assert lib.sv_beam_step(*a) == -6
    a = list(base)
    a[2] = 33   # beams > 32
    a[30] = 1 << 30
    assert lib.sv_beam_step(*a) == -3
    a = list(base)
    a[12] = 65  # num_picks > 64
    a[30] = 1 << 30
    assert lib.sv_beam_step(*a) == -3


def test_loop_guard_rejects_invalid_arguments(sv):
    lib = sv._lib.lib()
    assert lib.sv_loop_guard(None, 4, 1, 10, 8, 64, 3, 8, None) == -1
    assert lib.sv_loop_guard(8, 2, 1, 10, 8, 64, 3, 8, None) == -2
    assert lib.sv_loop_guard(8, 4, 1, 10, 8, 2000, 3, 8, None) == -4
    assert lib.sv_loop_guard(8, 4, 0, 10, 8, 64, 3, 8, None) == -3


def test_kv_reorder_rejects_invalid_arguments(sv):
    """sv_kv_reorder(keys, values, elem_bytes, layers, beams, heads, length, head_dim,
    stride_layer, stride_beam, stride_head, stride_slot, parents, out_status, stream):
    every rejection below returns before any CUDA call."""
    lib = sv._lib.lib()
    base = [16, 16, 2, 24, 2, 1, 100, 128, 2 * 4096 * 128, 4096 * 128, 0, 128, 16, None, None]

    def call(**kw):
        a = list(base)
        for k, v in kw.items():
            a[int(k[1:])] = v
        return lib.sv_kv_reorder(*a)

    assert call(a0=None) == -1 and call(a12=None) == -1
    assert call(a2=3) == -2
    assert call(a4=9) == -3 and call(a4=0) == -3 and call(a3=0) == -3 and call(a6=-1) == -3
    assert call(a3=70000) == -3                        # layers * heads > 65535
    assert call(a6=1 << 27, a7=128) == -3               # length * head_dim * elem_bytes >= 2^34
    assert call(a7=4) == -5                             # head_dim * elem_bytes not a multiple of 16
    assert call(a11=12) == -5 and call(a0=24) == -5     # stride / pointer alignment
    assert call(a6=0) == 0                              # nothing to copy: no launch


def test_beam_advance_rejects_invalid_arguments(sv):
    """sv_beam_advance(picks, pick_scores, n_picks, status, beams, vocab, num_picks,
    step, last, stop_ids, n_stop, eos_id, tails_in, tails_out, running_out,
    parents_out, tokens_out, seen_in, seen_out, seen_stride_words, hist_in, hist_out,
    hist_stride, whash_in, whash_out, guard_table, guard_entries, window, stream):
    rejections return before any CUDA call."""
    lib = sv._lib.lib()
    base = [16, 16, 16, 16, 2, 100, 4, 3, 0, 16, 2, -1, 16, 32, 16, 16, 16, 64, 128, 4, 256, 512, 8,
            1024, 1040, 2048, 64, 64, None]

    def call(**kw):
        a = list(base)
        for k, v in kw.items():
            a[int(k[1:])] = v
        return lib.sv_beam_advance(*a)

    assert call(a0=None) == -1 and call(a14=None) == -1 and call(a16=None) == -1
    assert call(a9=None) == -1 and call(a12=None) == -1            # stop ids without their tails
    assert call(a18=None) == -1 and call(a21=None) == -1           # one of a pair
    assert call(a6=65) == -3 and call(a4=5) == -3 and call(a10=17) == -3 and call(a7=-1) == -3
    assert call(a19=3) == -3                                       # seen stride < ceil(vocab / 32)
    assert call(a13=16) == -1 and call(a21=256) == -1              # in place
    assert call(a22=3) == -1                                       # history row shorter than step + 1
    assert call(a18=70) == -1                                      # seen_out overlaps seen_in
    assert call(a20=None, a21=None) == -1                          # the guard needs the histories
    assert call(a24=1024) == -1 and call(a23=None) == -1           # rolling hashes in place / missing
    assert call(a26=48) == -3 and call(a27=0) == -3 and call(a27=1025) == -3
    assert call(a25=2052) == -5                                    # table not 8-byte aligned


def test_loop_guard_incremental_rejects_invalid_arguments(sv):
    """sv_loop_guard_incremental(table, entries, tokens, token_bytes, insert_from,
    length, window, repeats, out_verdict, out_status, stream)."""
    lib = sv._lib.lib()
    base = [64, 1024, 128, 4, 0, 200, 64, 3, 16, None, None]

    def call(**kw):
        a = list(base)
        for k, v in kw.items():
            a[int(k[1:])] = v
        return lib.sv_loop_guard_incremental(*a)

    assert call(a0=None) == -1 and call(a2=None) == -1 and call(a8=None) == -1
    assert call(a3=2) == -2
    assert call(a1=1000) == -3 and call(a1=1) == -3 and call(a4=201) == -3 and call(a5=-1) == -3
    assert call(a6=0) == -4 and call(a6=1025) == -4 and call(a7=0) == -4
    assert call(a2=130) == -5 and call(a0=68) == -5


def test_torch_extension_loads_and_checks_tensors(sv):
    """The thin PyTorch extension (sv_torch) loads beside the C library and rejects
    non-CUDA tensors with a clear error before any CUDA call."""
    import torch
    ext = sv.ops._ext()
    assert ext.abi_version() == sv._lib.lib().sv_abi_version()
    for name in ("sample_step", "beam_step", "beam_advance", "kv_reorder", "loop_guard", "loop_guard_incremental"):
        assert callable(getattr(ext, name))
    x = torch.zeros(2, 64)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ext.loop_guard(torch.zeros(2, 64, dtype=torch.int32), 2, 64, torch.zeros(2, dtype=torch.int32), 8, 3,
                       torch.zeros(2, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ext.sample_step(x, 2, 64, 64, None, 0, 0, None, 0, torch.zeros(2), 1.5, 0.9, 50, 1, 3.1,
                        torch.zeros(2, dtype=torch.int64), None, None, None, None, 0, None, 0, 64,
                        torch.zeros(2, dtype=torch.int32), None, 0, 0)
