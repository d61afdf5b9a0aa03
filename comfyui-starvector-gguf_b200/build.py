"""Build the sm_100a C-ABI library and its thin PyTorch extension in-tree.

    python comfyui-starvector-gguf_b200/build.py [--force] [--verbose]

nvcc compiles csrc/*.cu for sm_100a (-gencode arch=compute_100a,code=sm_100a) into
libstarvector_sampling.so next to this file, with the CUDA runtime linked
statically so the library does not depend on the runtime version torch ships.
g++ then compiles ext/sv_torch.cpp against torch's headers into the extension
module sv_torch (next to this file), linked to that library: the tensor-level
functions ops.py calls on the hot path.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libstarvector_sampling.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-cudart", "static", "-I", INCLUDE, "-o", LIB + ".tmp", *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


EXT_SRC = os.path.join(HERE, "ext", "sv_torch.cpp")


def ext_path() -> str:
    import sysconfig
    return os.path.join(HERE, "sv_torch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False) -> str:
    """The PyTorch extension module (needs the C-ABI library first)."""
    import sysconfig

    import torch
    out = ext_path()
    deps = [EXT_SRC, LIB] + glob.glob(os.path.join(INCLUDE, "*.h"))
    if not force and os.path.exists(out) and all(os.path.getmtime(p) <= os.path.getmtime(out) for p in deps):
        return out
    tdir = os.path.dirname(torch.__file__)
    tinc, tlib = os.path.join(tdir, "include"), os.path.join(tdir, "lib")
    cuda_home = os.environ.get("CUDA_HOME", os.path.dirname(os.path.dirname(NVCC)))
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=sv_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", tinc, "-I", os.path.join(tinc, "torch", "csrc", "api", "include"),
           "-I", os.path.join(cuda_home, "include"), "-I", sysconfig.get_paths()["include"], "-I", INCLUDE,
           EXT_SRC, "-o", out + ".tmp",
           "-L", tlib, "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
           "-L", HERE, "-l:" + os.path.basename(LIB), "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + tlib]
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
    print(build_ext(force="--force" in sys.argv))
