"""ctypes binding of libstarvector_sampling.so (the C ABI in include/starvector_sampling.h).

There is no fallback: if the library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstarvector_sampling.so")

SV_OK = 0
SV_E_ARG, SV_E_DTYPE, SV_E_SHAPE, SV_E_RANGE, SV_E_ALIGN, SV_E_WORKSPACE, SV_E_CUDA = range(-1, -8, -1)
ST_OK, ST_NAN, ST_POSINF, ST_ALLNEGINF, ST_HISTORY, ST_TIMEOUT, ST_SHARD_OVERFLOW, ST_GUARD_FULL = range(8)
F32, F16, BF16 = 0, 1, 2
HIST_NONE, HIST_IDS32, HIST_IDS64, HIST_MASK8, HIST_BITS32 = range(5)
DENSE_NONE, DENSE_SCORES, DENSE_PROBS = range(3)
FLAG_FORCE_GENERAL = 1
FLAG_CLUSTER = 2
FLAG_STREAM = 4
FLAG_TEST_WAIT_TIMEOUT = 8

_P, _I32, _I64, _D, _SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_double, C.c_size_t

_SIGNATURES = {
    "sv_sample_step": (_I32, [_P, _I32, _I32, _I32, _I64, _P, _I32, _I64, _P, _I32, _P, _D, _D, _I32, _I32, _D,
                              _P, _P, _P, _P, _P, _I32, _P, _I32, _I64, _P, _P, _I64, _I32, _P]),
    "sv_beam_workspace_bytes": (_SZ, [_I32, _I32]),
    "sv_beam_step": (_I32, [_P, _I32, _I32, _I32, _I64, _P, _I32, _I64, _P, _I32, _P, _P, _I32, _D, _D, _I32, _I32,
                            _D, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _I64, _P, _SZ, _I32, _P]),
    "sv_loop_guard": (_I32, [_P, _I32, _I32, _I64, _P, _I32, _I32, _P, _P]),
    "sv_penalize": (_I32, [_P, _I32, _I32, _I32, _I64, _P, _I32, _I64, _D, _P, _I64, _P]),
    "sv_seen_update": (_I32, [_P, _I32, _I64, _P, _I32, _P]),
    "sv_seen_reorder": (_I32, [_P, _P, _I32, _I32, _I64, _P, _P, _P]),
    "sv_merge_shards": (_I32, [_P, _I32, _I32, _I32, _P, _D, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P]),
    "sv_pack_slice": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _P, _P]),
    "sv_beam_slice_stats": (_I32, [_P, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P]),
    "sv_beam_slice_logprobs": (_I32, [_P, _I32, _I32, _I32, _I64, _P, _P, _P, _I64, _P]),
    "sv_merge_beam_shards_workspace_bytes": (_SZ, [_I32, _I32, _I32]),
    "sv_merge_beam_shards": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _D, _I32, _I32, _P, _SZ,
                                    _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P]),
    "sv_merge_slices": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _D, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P]),
    "sv_merge_beam_slices": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _D, _I32, _I32, _P, _SZ,
                                    _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P]),
    "sv_kv_reorder": (_I32, [_P, _P, _I32, _I32, _I32, _I32, _I64, _I32, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "sv_beam_advance": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _I32, _I64, _P, _P, _P, _P, _P, _P,
                               _P, _I64, _P, _P, _I64, _P, _P, _P, _I64, _I32, _P]),
    "sv_loop_guard_incremental": (_I32, [_P, _I64, _P, _I32, _I64, _I64, _I32, _I32, _P, _P, _P]),
    "sv_error_string": (C.c_char_p, [_I32]),
    "sv_abi_version": (_I32, []),
}

_lib = None


def lib():
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"StarVector B200 sampling library not built: {LIB_PATH} is missing "
                               "(run comfyui-starvector-gguf_b200/build.py)")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def error_string(code: int) -> str:
    return lib().sv_error_string(int(code)).decode()


def check(rc: int, what: str) -> None:
    """Turn a negative return code into the exception the reference would raise."""
    if rc == SV_OK:
        return
    msg = f"{what}: {error_string(rc)} (code {rc})"
    if rc in (SV_E_RANGE,):
        raise ValueError(msg)
    raise RuntimeError(msg)
