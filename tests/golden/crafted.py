"""Crafted variants of a synthetic GGUF model -- TEST INFRASTRUCTURE.

The greedy argmax must follow ss_argmax (SlipStream/src/core/tensor.c:318-328)
exactly, including its edge cases, and those only appear in the logits when the
lm_head rows are made for them.  ``make_crafted(case, src, dst)`` copies a
synthetic GGUF and rewrites the fp16 block scales (and for some cases the
blocks) of ``output.weight``:

* ``nan0``   -- row 0's first block scale is NaN, so logit 0 is NaN: the
  reference never moves off index 0.
* ``zeros``  -- every row's scales are +0 except rows 3 and 7, copies of row
  100: logits are +-0 except two equal values (a tie between rows 3 and 7 if
  they are the largest, else a tie between the zeros).
* ``allzero`` -- every scale is +0 (logits +-0 only: index 0 by the tie rule).
* ``negzero`` -- every scale is -0 except rows 5 and 9, copies of row 100
  with their scales negated (so the two equal logits have the opposite sign to
  those of the ``zeros`` case).

``argmax_arrays()`` gives seeded edge-case inputs of the argmax itself.

Used by tests/golden/make_golden.py (expectations from the reference build)
and the GPU tests (the same bytes on the GPU host).
"""
from __future__ import annotations

import shutil
import struct

import numpy as np

CASES = ("nan0", "zeros", "allzero", "negzero")

_SCALAR = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
_BLOCK = {2: (18, 32), 8: (34, 32)}  # type -> (bytes, weights) per block


def _skip_value(f, vtype: int) -> None:
    if vtype in _SCALAR:
        f.read(_SCALAR[vtype])
    elif vtype == 8:
        (n,) = struct.unpack("<Q", f.read(8))
        f.read(n)
    elif vtype == 9:
        et, n = struct.unpack("<IQ", f.read(12))
        for _ in range(n):
            _skip_value(f, et)
    else:
        raise ValueError(f"unknown GGUF value type {vtype}")


def tensor_table(path: str) -> dict:
    """{name: (absolute data offset, ggml type, dims)} of a GGUF v3 file
    (data section aligned to 32 bytes, the synthetic writer's alignment)."""
    with open(path, "rb") as f:
        magic, version, nt, nkv = struct.unpack("<4sIQQ", f.read(24))
        if magic != b"GGUF" or version != 3:
            raise ValueError(f"{path}: not a GGUF v3 file")
        for _ in range(nkv):
            (klen,) = struct.unpack("<Q", f.read(8))
            f.read(klen)
            (vt,) = struct.unpack("<I", f.read(4))
            _skip_value(f, vt)
        infos = []
        for _ in range(nt):
            (nlen,) = struct.unpack("<Q", f.read(8))
            name = f.read(nlen).decode()
            (nd,) = struct.unpack("<I", f.read(4))
            dims = struct.unpack(f"<{nd}Q", f.read(8 * nd))
            ttype, off = struct.unpack("<IQ", f.read(12))
            infos.append((name, dims, ttype, off))
        base = (f.tell() + 31) // 32 * 32
    return {n: (base + off, t, dims) for n, dims, t, off in infos}


def make_crafted(case: str, src: str, dst: str) -> None:
    if case not in CASES:
        raise ValueError(case)
    shutil.copyfile(src, dst)
    off, ttype, dims = tensor_table(dst)["output.weight"]
    bb, bw = _BLOCK[ttype]
    cols, rows = int(dims[0]), int(dims[1])
    nb = cols // bw
    m = np.memmap(dst, dtype=np.uint8, mode="r+", offset=off, shape=(rows, nb, bb))
    scale = m[:, :, 0:2].view(np.uint16)[..., 0]  # [rows, nb] fp16 bits
    if case == "nan0":
        scale[0, 0] = 0x7E00
    elif case in ("zeros", "allzero"):
        keep = {3: 100, 7: 100} if case == "zeros" else {}
        blocks = {r: np.array(m[s]) for r, s in keep.items()}
        scale[:, :] = 0x0000
        for r, b in blocks.items():
            m[r] = b
    else:  # negzero
        blocks = {r: np.array(m[100]) for r in (5, 9)}
        scale[:, :] = 0x8000
        for r, b in blocks.items():
            m[r] = b
            m[r, :, 1] ^= 0x80  # flip the sign bit of every block scale
    m.flush()
    del m


def argmax_arrays() -> dict:
    """Edge cases of ss_argmax's rule (tensor.c:318-328): NaN first or later,
    -0.0 against +0.0, ties, infinities, and large multi-block arrays."""
    nan, inf = np.float32(np.nan), np.float32(np.inf)
    small = [
        [nan, 1.0, 2.0], [1.0, nan, 3.0, nan], [-0.0, 0.0, -1.0], [-1.0, 0.0, -0.0],
        [-1.0, -0.0, 0.0], [nan] * 5, [-inf, nan, -inf], [3.0, 5.0, 5.0, 1.0],
        [-inf, -inf], [inf, inf, 1.0], [-2.0, -0.0, -3.0, 0.0, -0.0], [7.0],
    ]
    cases = {f"small{i}": np.array(a, np.float32) for i, a in enumerate(small)}
    rng = np.random.default_rng(77)
    n = 1 << 22  # the allocation-free argmax's maximum
    big = -np.abs(rng.standard_normal(n)).astype(np.float32) - 1.0
    a = big.copy()
    a[1000], a[3_000_000] = -0.0, 0.0  # only zeros are the maximum: the first wins
    cases["big_zero_tie"] = a
    a = big.copy()
    a[0] = nan
    a[12345] = 5.0
    cases["big_nan0"] = a
    a = big.copy()
    a[[7, 4_000_000]] = nan
    a[[2_500_000, 4_194_303]] = 9.0
    cases["big_tie_end"] = a
    return cases
