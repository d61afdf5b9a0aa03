"""B200-native (sm_100a) decode-sampling step of ComfyUI-StarVector-GGUF.

Layout:
  csrc/               CUDA kernels and the extern "C" layer (include/starvector_sampling.h)
  build.py            nvcc build of libstarvector_sampling.so, in-tree
  _lib.py             ctypes binding of the C ABI (no fallback: a missing library raises)
  ops.py              torch-tensor wrappers: sample_step, beam_step, loop_guard, penalize, ...
  runtime_shared.py   drop-in for the reference's sampling functions (_sample, _beam_sample & co.)
  sharded.py          row-sharded and vocabulary-sharded multi-GPU sampling (torch.distributed)

The directory name is not a Python identifier (it is a ComfyUI custom-node folder);
load it by path, e.g. through __graft_entry__.load_package(), which registers it as
`starvector_b200`.
"""
from . import _lib, sharded
from .ops import (beam_advance, beam_step, beam_workspace, kv_reorder, loop_guard, merge_beam_shards, merge_shards,
                  penalize, sample_step, seen_bitmap, seen_reorder, seen_update)

__all__ = ["sample_step", "beam_step", "beam_workspace", "beam_advance", "kv_reorder", "loop_guard",
           "merge_beam_shards", "merge_shards", "penalize", "seen_bitmap", "seen_reorder", "seen_update", "sharded"]
