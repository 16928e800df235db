"""In-tree build of the native libraries.

* ``phonemap_b200/lib/libslipstream_cuda.so`` -- the CUDA backend (sm_100a
  kernels + the C ABI declared in ``include/slipstream_cuda.h``), built with
  ``nvcc -gencode arch=compute_100a,code=sm_100a``.
* ``phonemap_b200/lib/libss_synth.so`` -- the synthetic GGUF writer.

The outputs are git-ignored but live inside the tree so that they travel with a
snapshot of the repository to a GPU host.  ``python -m phonemap_b200.build``
builds everything.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
INCLUDE = os.path.join(ROOT, "include")

CUDA_LIB = os.path.join(LIBDIR, "libslipstream_cuda.so")
SYNTH_LIB = os.path.join(LIBDIR, "libss_synth.so")

CUDA_SOURCES = ["ss_cuda_api.cu", "noalloc_argmax.cu", "sample.cu", "quant.cu"]
CUDA_HEADERS = ["common.cuh", "gemv.cuh", "attention.cuh", "misc_kernels.cuh",
                "step_kernel.cuh", "qgemm.cuh", "qgemm_host.inc", "batch_kernels.cuh",
                "batch_host.inc", "tp_nccl.h", "gguf_view.h", "sample.h", "quant.h",
                "ss_cuda_internal.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_synth(force: bool = False) -> str:
    src = os.path.join(CSRC, "synth_gguf.c")
    if force or _stale(SYNTH_LIB, [src]):
        os.makedirs(LIBDIR, exist_ok=True)
        subprocess.run(["gcc", "-std=gnu11", "-O2", "-fopenmp", "-fPIC", "-shared", src,
                        "-o", SYNTH_LIB, "-lm"], check=True)
    return SYNTH_LIB


def build_cuda(force: bool = False, extra: list[str] | None = None) -> str:
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in CUDA_HEADERS] + [
        os.path.join(INCLUDE, "slipstream_cuda.h")]
    if force or extra or _stale(CUDA_LIB, deps):
        os.makedirs(LIBDIR, exist_ok=True)
        cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
               "-I", INCLUDE, "-I", CSRC, *srcs, "-o", CUDA_LIB,
               "-ldl", "-lpthread", *(extra or [])]
        subprocess.run(cmd, check=True)
    return CUDA_LIB


def build_all(force: bool = False) -> list[str]:
    return [build_synth(force), build_cuda(force)]


if __name__ == "__main__":
    for p in build_all(force="--force" in sys.argv):
        print(p)
