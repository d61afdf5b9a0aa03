"""sv_beam_step_noalloc, the beam step for callers that cannot allocate device
memory (a host application that owns the GPU's memory pool, or a loop that must
not allocate during a step), checked through the C ABI against sv_beam_step with
its own workspace: the same picks, scores, counts and statuses bit for bit (the
tolerance of every beam parity test here), on two calls in a row.

This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import bench

pytestmark = pytest.mark.gpu
DEV = "cuda"

_P, _I32, _I64, _D = C.c_void_p, C.c_int32, C.c_int64, C.c_double
_ARGS = [_P, _I32, _I32, _I32, _I64, _P, _I32, _I64, _P, _I32, _P, _P, _I32, _D, _D, _I32, _I32, _D,
         _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _I64, _I32, _P]


def noalloc_fn(sv):
    fn = sv._lib.lib().sv_beam_step_noalloc
    fn.argtypes = _ARGS
    fn.restype = _I32
    return fn


def call_noalloc(sv, x, rs, u, hist, npick, cap):
    B, V = x.shape
    dt = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[x.dtype]
    out = dict(picks=torch.full((npick,), -1, dtype=torch.int64, device=DEV),
               scores=torch.zeros(npick, device=DEV), n=torch.zeros(1, dtype=torch.int32, device=DEV),
               status=torch.zeros(1, dtype=torch.int32, device=DEV),
               kept_count=torch.zeros(B, dtype=torch.int32, device=DEV),
               kept_idx=torch.full((B, cap), -1, dtype=torch.int32, device=DEV),
               kept_logprob=torch.zeros((B, cap), device=DEV), kept_prob=torch.zeros((B, cap), device=DEV))
    rc = noalloc_fn(sv)(x.data_ptr(), dt, B, V, x.stride(0), hist.data_ptr(), 1, hist.stride(0), None, hist.shape[1],
                        rs.data_ptr(), u.data_ptr(), npick, 1.5, 0.9, 50, 2, 3.1,
                        out["picks"].data_ptr(), out["scores"].data_ptr(), out["n"].data_ptr(),
                        out["status"].data_ptr(), out["kept_count"].data_ptr(), out["kept_idx"].data_ptr(),
                        out["kept_logprob"].data_ptr(), out["kept_prob"].data_ptr(), cap, None, 0, 0,
                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, sv._lib.error_string(rc)
    return out


@pytest.mark.parametrize("cfg,dtype", [(bench.cfg2, torch.float32), (bench.cfg3, torch.bfloat16)],
                         ids=["cfg2-2beams-f32", "cfg3-8beams-bf16"])
def test_noalloc_matches_workspace_version_twice(sv, cfg, dtype):
    for call, seed in enumerate((11, 12)):
        d = cfg(seed=seed)
        x = torch.from_numpy(d["logits"]).to(DEV).to(dtype)
        rs = torch.from_numpy(d["running"]).to(DEV)
        u = torch.from_numpy(d["uniforms"]).to(DEV)
        h = torch.from_numpy(d["history"]).to(DEV)
        B = x.shape[0]
        ref = sv.beam_step(x, rs, u, history=h, num_picks=2 * B, out_capacity=64)
        got = call_noalloc(sv, x, rs, u, h, 2 * B, 64)
        torch.cuda.synchronize()
        assert int(ref["status"][0]) == 0, call
        for k in ("picks", "scores", "n", "status", "kept_count", "kept_idx", "kept_logprob", "kept_prob"):
            assert torch.equal(got[k], ref[k]), (call, k)


def test_noalloc_rejects_sizes_beyond_its_scratch(sv):
    x = torch.zeros((16, 40000), device=DEV)  # 16 x 40000 > 524271 entries
    rs = torch.zeros(16, device=DEV)
    u = torch.zeros(32, device=DEV)
    h = torch.zeros((16, 1), dtype=torch.int32, device=DEV)
    out = torch.zeros(64, dtype=torch.int64, device=DEV)
    rc = noalloc_fn(sv)(x.data_ptr(), 0, 16, 40000, 40000, h.data_ptr(), 1, 1, None, 1, rs.data_ptr(),
                        u.data_ptr(), 32, 1.5, 0.9, 50, 2, 3.1, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                        out.data_ptr(), None, None, None, None, 0, None, 0, 0, None)
    assert rc == -8
    assert "fixed scratch" in sv._lib.error_string(rc)
