"""Shared pytest setup: the `gpu` marker and the repository root on sys.path.

GPU tests are marked `@pytest.mark.gpu`; `pytest -m "not gpu"` runs everything
that needs no GPU (the oracle against the golden vectors, host logic, the C-ABI
library's symbol table, multi-process gloo tests).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")


@pytest.fixture(scope="session")
def sv():
    """The product package (comfyui-starvector-gguf_b200) loaded as `starvector_b200`;
    the C library and its torch extension are built first when either is missing
    (a fresh checkout)."""
    import glob

    import __graft_entry__
    pkg = __graft_entry__.PKG_DIR
    if not (os.path.exists(os.path.join(pkg, "libstarvector_sampling.so")) and glob.glob(os.path.join(pkg, "sv_torch*.so"))):
        __graft_entry__.build()
    return __graft_entry__.load_package()
