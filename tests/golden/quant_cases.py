"""Seeded GGUF blocks of every type the reference dequantizes -- TEST
INFRASTRUCTURE.

``blocks(type)`` gives (bytes, n values) for a type of SlipStream/src/core/
quantize.c:389-442: random quant bits, and scale / min fields set to float16
(or, for Q8_1, float32) values drawn from a normal distribution, with some
blocks carrying edge scales (zero, negative zero, subnormal, the largest
float16).  No NaN or infinite scale: the result's NaN payload would depend on
the machine.  ``q4k_matrix()`` is a Q4_K matrix and vector for the matvec
twin of ss_metal_matvec_q4_K.  Used by tests/golden/make_golden.py (the
reference's outputs), tests/test_oracle_quant.py and tests/test_gpu_quant.py.
"""
from __future__ import annotations

import numpy as np

# ggml type -> (bytes per block, values per block, offsets of float16 fields,
# offsets of float32 fields)
TYPES = {
    1: (2, 1, (0,), ()),            # F16
    2: (18, 32, (0,), ()),          # Q4_0
    3: (20, 32, (0, 2), ()),        # Q4_1
    6: (22, 32, (0,), ()),          # Q5_0
    7: (24, 32, (0, 2), ()),        # Q5_1
    8: (34, 32, (0,), ()),          # Q8_0
    9: (40, 32, (), (0, 4)),        # Q8_1
    10: (84, 256, (80, 82), ()),    # Q2_K
    11: (110, 256, (108,), ()),     # Q3_K
    12: (144, 256, (0, 2), ()),     # Q4_K
    13: (176, 256, (0, 2), ()),     # Q5_K
    14: (210, 256, (208,), ()),     # Q6_K
}
NAMES = {1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1", 10: "Q2_K",
         11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}
EDGE = np.array([0.0, -0.0, 6.0e-8, -3.0e-6, 65504.0, 1.0, -1.0], np.float16)


def blocks(t: int, nblk: int = 40, seed: int = 0) -> tuple[np.ndarray, int]:
    ts, bs, f16, f32 = TYPES[t]
    rng = np.random.default_rng(1000 * t + seed)
    if t == 1:  # plain float16 values, edge ones included
        v = (rng.standard_normal(nblk * 32) * 0.5).astype(np.float16)
        v[: EDGE.size] = EDGE
        return v.view(np.uint8).copy(), v.size
    raw = rng.integers(0, 256, size=(nblk, ts), dtype=np.uint8)
    for off in f16:
        s = (rng.standard_normal(nblk) * 0.02).astype(np.float16)
        s[: EDGE.size] = EDGE[: min(EDGE.size, nblk)]
        raw[:, off:off + 2] = s.view(np.uint8).reshape(nblk, 2)
    for off in f32:
        s = (rng.standard_normal(nblk) * 0.02).astype(np.float32)
        s[0] = 0.0
        raw[:, off:off + 4] = s.view(np.uint8).reshape(nblk, 4)
    return raw.reshape(-1), nblk * bs


def q4k_matrix(rows: int = 48, cols: int = 1024, seed: int = 5):
    """A Q4_K matrix [rows][cols / 256 blocks] (GGUF row order) and x[cols]."""
    raw, _ = blocks(12, rows * cols // 256, seed)
    x = np.random.default_rng(seed + 1).standard_normal(cols).astype(np.float32)
    return raw, x
