"""phonemap_b200 -- B200-native (sm_100a) CUDA backend for SlipStream's decode path.

SlipStream is the on-device GGUF inference engine inside harrisonfar123/PhoneMap.
This package holds its per-token decode loop (Q4_0/Q8_0 dequant-matvec, RMSNorm,
RoPE, int8-KV GQA attention, SwiGLU, lm_head + greedy argmax) as hand-written
CUDA kernels behind a C ABI (include/slipstream_cuda.h), plus:

* ``runtime``  -- ctypes binding of that C ABI (``CudaModel``);
* ``configs``  -- the benchmark model shapes;
* ``synth``    -- the seeded synthetic GGUF writer used for benchmarks/tests;
* ``build``    -- in-tree nvcc build of the native libraries.
"""
from . import configs  # noqa: F401
