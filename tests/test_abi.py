"""The C ABI library loads and exports every entry point include/slipstream_cuda.h
declares (no GPU calls)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from phonemap_b200 import build, runtime

HEADER = os.path.join(build.INCLUDE, "slipstream_cuda.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ss_cuda_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(runtime.EXPORTED)


def test_library_exports_every_declared_symbol():
    if not os.path.exists(build.CUDA_LIB):
        build.build_cuda()
    lib = ctypes.CDLL(build.CUDA_LIB)
    missing = [f for f in declared_functions() if not hasattr(lib, f)]
    assert not missing, f"not exported: {missing}"
    assert lib.ss_cuda_abi_version() == 1
    lib.ss_cuda_should_use_gpu.restype = ctypes.c_bool
    assert lib.ss_cuda_should_use_gpu(1, 1)


def test_built_for_sm100a_only():
    """The build compiles for sm_100a and nothing else (the loaded kernels'
    binary version is checked on the GPU: tests/test_gpu_kernels.py)."""
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_integration_build_links_backend():
    """oracle/_ref/libss_ref_cuda.so (the reference with the INTEGRATION.md
    hook, where the reference sources were present at build time) loads and
    binds this library's matvec entry points."""
    import ctypes

    import oracle
    path = os.path.join(oracle.REF_DIR, "libss_ref_cuda.so")
    if not os.path.exists(path):
        pytest.skip("integration build absent")
    lib = ctypes.CDLL(path)
    assert hasattr(lib, "ssr_attach_cuda") and hasattr(lib, "ssr_forward")
