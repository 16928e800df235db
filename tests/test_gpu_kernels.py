"""GPU: dequantisation bit-exactness and the op-level (Metal-twin) matvecs,
called through the C ABI (include/slipstream_cuda.h)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err

pytestmark = pytest.mark.gpu

Q4, Q8 = 2, 8


@pytest.mark.parametrize("kind,t", [("q4_0", Q4), ("q8_0", Q8)])
def test_dequant_blocks_bitexact(kind, t):
    """Seeded + edge blocks (zero/negative/subnormal/max fp16 scales, all-0x0 /
    all-0xF nibbles) dequantised on the device == the reference's
    ss_dequantize (quantize.c:60-72, :139-149), bit for bit."""
    g = load_golden("ops")
    raw, want = g[f"{kind}_raw"], g[f"{kind}_deq"]
    got = runtime.dequantize_blocks(t, raw, want.size)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("flags", [0, runtime.FLAG_MULTI_KERNEL], ids=["tiled", "row-interleaved"])
@pytest.mark.parametrize("name", ["tiny", "tiny-q8"])
def test_uploaded_tensors_dequantise_bitexact(name, flags):
    """Every repacked weight tensor in HBM decodes to exactly the reference
    dequantisation of the GGUF bytes (covers upload + repack + decode), in both
    device layouts: tiled (persistent step) and row-interleaved (multi-kernel)."""
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    ops = oracle.oracle_ops()
    import ctypes
    from tests.golden.fingerprint import gguf_fingerprint  # noqa: F401
    with runtime.CudaModel(path, cfg.ctx, flags=flags) as m:
        assert m.stats()["persistent"] == (0 if flags else 1)
        raw = np.fromfile(path, np.uint8)
        # locate tensors through the oracle's own loader: re-read offsets
        tensors = _tensor_table(path)
        for tname, (off, rows, cols, typ) in tensors.items():
            if typ not in (Q4, Q8):
                continue
            n = rows * cols
            want = np.empty(n, np.float32)
            blob = np.ascontiguousarray(raw[off: off + n // 32 * (18 if typ == Q4 else 34)])
            ops.sso_dequantize(blob.ctypes.data, want.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                               n, typ)
            got = m.dequantize_tensor(tname, rows, cols).reshape(-1)
            np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=tname)


def _tensor_table(path: str) -> dict:
    """name -> (absolute offset, rows, cols, type) from the GGUF header."""
    import struct
    data = open(path, "rb").read(1 << 20)
    pos = 24
    _, _, n_t, n_kv = struct.unpack_from("<IIQQ", data)

    def rstr(p):
        (ln,) = struct.unpack_from("<Q", data, p)
        return data[p + 8: p + 8 + ln].decode(), p + 8 + ln
    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    for _ in range(n_kv):
        _, pos = rstr(pos)
        (t,) = struct.unpack_from("<I", data, pos)
        pos += 4
        if t == 8:
            _, pos = rstr(pos)
        else:
            pos += sizes[t]
    out = {}
    for _ in range(n_t):
        name, pos = rstr(pos)
        (nd,) = struct.unpack_from("<I", data, pos)
        pos += 4
        dims = struct.unpack_from("<" + "Q" * nd, data, pos)
        pos += 8 * nd
        typ, off = struct.unpack_from("<IQ", data, pos)
        pos += 12
        out[name] = (off, dims[1] if nd > 1 else 1, dims[0], typ)
    base = (pos + 31) & ~31
    return {k: (v[0] + base, v[1], v[2], v[3]) for k, v in out.items()}


@pytest.mark.parametrize("kind,t", [("q4_0", Q4), ("q8_0", Q8)])
def test_op_matvec_vs_reference(kind, t):
    """ss_cuda_matvec_q4_0 / _q8_0 (twins of ss_metal_matvec_q4_0) vs the
    reference dequant-matvec on the golden blocks; fp32, different summation
    order: |err| <= 1e-5 of the row norm."""
    g = load_golden("ops")
    raw, x, want = g[f"{kind}_raw"], g[f"{kind}_x"], g[f"{kind}_mv"]
    rows, cols = want.size, x.size
    with runtime.CudaModel(None) as m:
        got = m.matvec(raw, x, rows, cols, t)
        got2 = m.matvec(raw, x, rows, cols, t)  # cached device copy
    deq = g[f"{kind}_deq"].reshape(rows, cols).astype(np.float64)
    scale = np.abs(deq).dot(np.abs(x.astype(np.float64))) + 1e-30
    assert np.all(np.abs(got - want) <= 1e-5 * scale)
    np.testing.assert_array_equal(got, got2)


@pytest.mark.parametrize("rows,cols,t", [(4096, 4096, Q4), (11008, 4096, Q4), (4096, 11008, Q4),
                                         (1000, 2048, Q8), (32, 32, Q4), (7, 96, Q8), (5, 64, Q4)])
def test_op_matvec_shapes(rows, cols, t):
    """Full-size and ragged shapes (rows not a multiple of 4, a single block per
    row) against the oracle's sequential dequant-matvec."""
    rng = np.random.default_rng(rows * 7 + cols)
    nb = rows * cols // 32
    bsz = 18 if t == Q4 else 34
    blocks = rng.integers(0, 256, size=(nb, bsz), dtype=np.uint8)
    blocks[:, 0:2] = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    raw = np.ascontiguousarray(blocks.reshape(-1))
    x = rng.standard_normal(cols).astype(np.float32)
    ops = oracle.oracle_ops()
    import ctypes
    F = ctypes.POINTER(ctypes.c_float)
    want = np.empty(rows, np.float32)
    ops.sso_dequant_matvec(want.ctypes.data_as(F), raw.ctypes.data, x.ctypes.data_as(F), rows, cols, t)
    deq = np.empty(rows * cols, np.float32)
    ops.sso_dequantize(raw.ctypes.data, deq.ctypes.data_as(F), rows * cols, t)
    scale = np.abs(deq.reshape(rows, cols).astype(np.float64)).dot(np.abs(x.astype(np.float64)))
    with runtime.CudaModel(None) as m:
        got = m.matvec(raw, x, rows, cols, t)
    assert np.all(np.abs(got.astype(np.float64) - want) <= 2e-6 * scale + 1e-30)


@pytest.mark.parametrize("t", [Q4, Q8])
def test_op_matvec_extreme_activations(t):
    """Activations the block fixed-point conversion must survive: all-zero
    blocks, one dominant element per block, values down to 1e-20, mixed signs,
    exact powers of two.  Bound: each activation is represented to 2^-23 of its
    block's max |x|, the integer dot is exact, then two fp32 roundings."""
    rows, cols = 64, 1024
    rng = np.random.default_rng(99 + t)
    nb = rows * cols // 32
    bsz = 18 if t == Q4 else 34
    blocks = rng.integers(0, 256, size=(nb, bsz), dtype=np.uint8)
    blocks[:, 0:2] = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    raw = np.ascontiguousarray(blocks.reshape(-1))
    x = rng.standard_normal(cols).astype(np.float32)
    x[0:32] = 0.0                                   # empty block
    x[32:64] = 1e-6 * x[32:64]
    x[40] = 300.0                                   # one dominant element
    x[64:96] = np.float32(2.0) ** rng.integers(-30, 30, 32).astype(np.float32)
    x[96:128] = 1e-20 * x[96:128]                   # tiny block
    x[128:160] = -x[128:160] * 1e4
    ops = oracle.oracle_ops()
    import ctypes
    F = ctypes.POINTER(ctypes.c_float)
    deq = np.empty(rows * cols, np.float32)
    ops.sso_dequantize(raw.ctypes.data, deq.ctypes.data_as(F), rows * cols, t)
    w = deq.reshape(rows, cols).astype(np.float64)
    xd = x.astype(np.float64)
    exact = w.dot(xd)
    blockmax = np.repeat(np.abs(xd).reshape(-1, 32).max(1), 32)
    bound = 2.0 ** -22 * np.abs(w).dot(blockmax) + 2e-7 * np.abs(w).dot(np.abs(xd)) + 1e-30
    with runtime.CudaModel(None) as m:
        got = m.matvec(raw, x, rows, cols, t).astype(np.float64)
    assert np.all(np.abs(got - exact) <= bound)


def test_op_batch_brackets():
    """begin/end batch (twins of ss_metal_begin/end_batch): outputs land at
    end_batch and equal the unbatched results."""
    g = load_golden("ops")
    raw, x = g["q4_0_raw"], g["q4_0_x"]
    rows, cols = g["q4_0_mv"].size, x.size
    with runtime.CudaModel(None) as m:
        ref1 = m.matvec(raw, x, rows, cols, Q4)
        ref2 = m.matvec(raw, x * 2, rows, cols, Q4)
        m.begin_batch()
        a = m.matvec(raw, x, rows, cols, Q4)
        b = m.matvec(raw, x * 2, rows, cols, Q4)
        m.end_batch()
    # inside a batch the arrays are filled at end_batch (ctypes wrote into them)
    np.testing.assert_array_equal(a, ref1)
    np.testing.assert_array_equal(b, ref2)


def test_loaded_kernels_are_sm100a():
    """The kernels the context runs were compiled for sm_100a
    (cudaFuncAttributes::binaryVersion 100, ss_cuda_stats[14])."""
    cfg = configs.get("tiny")
    with runtime.CudaModel(synth.ensure_gguf(cfg), cfg.ctx) as m:
        assert m.stats()["kernel_arch"] == 100
