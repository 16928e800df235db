"""The GGUF block types on the device: ss_cuda_dequantize for every type of
SlipStream's ss_dequantize (SlipStream/src/core/quantize.c:389-442) against
the reference's own values (tests/golden/quant.npz) and the oracle on more
seeds, bit for bit; ss_cuda_matvec_q4_K (twin of ss_metal_matvec_q4_K,
metal_backend.m:111-154) against the reference's dequant-matvec, fp32 in
another summation order: |err| <= 1e-5 of sum |w| |x| per row, as the other
op-level matvecs."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from phonemap_b200 import runtime
from tests.conftest import load_golden
from tests.golden import quant_cases as qc

pytestmark = pytest.mark.gpu
F32P = ctypes.POINTER(ctypes.c_float)
IDS = [qc.NAMES[t] for t in sorted(qc.TYPES)]


@pytest.mark.parametrize("t", sorted(qc.TYPES), ids=IDS)
def test_dequantize_matches_reference(t):
    g = load_golden("quant")
    raw = g[f"{qc.NAMES[t]}/blocks"]
    want = g[f"{qc.NAMES[t]}/values"]
    got = runtime.dequantize_blocks(t, raw, want.size)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # more blocks, another seed: against the oracle
    raw2, n2 = qc.blocks(t, nblk=3000, seed=9)
    ref = np.empty(n2, np.float32)
    oracle.oracle_ops().sso_dequantize(raw2.ctypes.data, ref.ctypes.data_as(F32P), n2, t)
    np.testing.assert_array_equal(runtime.dequantize_blocks(t, raw2, n2).view(np.uint32), ref.view(np.uint32))


def test_dequantize_errors():
    raw, n = qc.blocks(12)
    with pytest.raises(runtime.SSCudaError):
        runtime.dequantize_blocks(12, raw, 100)  # not a multiple of 256
    with pytest.raises(runtime.SSCudaError):
        runtime.dequantize_blocks(4, raw, 256)  # no such type in the reference


def _row_scale(raw, x, rows, cols):
    deq = np.empty(rows * cols, np.float32)
    oracle.oracle_ops().sso_dequantize(raw.ctypes.data, deq.ctypes.data_as(F32P), rows * cols, 12)
    return np.abs(deq.reshape(rows, cols).astype(np.float64)).dot(np.abs(x.astype(np.float64))) + 1e-30


def test_q4k_matvec_matches_reference():
    g = load_golden("quant")
    raw, x, want = g["q4k_mv/w"], g["q4k_mv/x"], g["q4k_mv/out"]
    with runtime.CudaModel(None) as m:
        got = m.matvec(raw, x, 48, 1024, runtime.Q4_K)
        got2 = m.matvec(raw, x, 48, 1024, runtime.Q4_K)  # the cached device copy
    assert np.all(np.abs(got - want) <= 1e-5 * _row_scale(raw, x, 48, 1024))
    np.testing.assert_array_equal(got, got2)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (11008, 4096), (4096, 11008 // 256 * 256), (7, 256)])
def test_q4k_matvec_shapes(rows, cols):
    """Full-size and ragged shapes against the oracle's sequential
    dequant-matvec, inside the batch brackets too."""
    raw, _ = qc.blocks(12, rows * cols // 256, seed=rows + cols)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    want = np.empty(rows, np.float32)
    oracle.oracle_ops().sso_dequant_matvec(want.ctypes.data_as(F32P), raw.ctypes.data, x.ctypes.data_as(F32P),
                                           rows, cols, 12)
    scale = _row_scale(raw, x, rows, cols)
    with runtime.CudaModel(None) as m:
        got = m.matvec(raw, x, rows, cols, runtime.Q4_K)
        assert np.all(np.abs(got - want) <= 1e-5 * scale)
        lib = runtime.load_library()
        out = np.full(rows, np.nan, np.float32)
        m.begin_batch()
        assert lib.ss_cuda_matvec_q4_K(m._h, runtime._f(out), raw.ctypes.data, runtime._f(x), rows, cols)
        m.end_batch()
        np.testing.assert_array_equal(out, got)
        assert not lib.ss_cuda_matvec_q4_K(m._h, runtime._f(out), raw.ctypes.data, runtime._f(x), rows, cols - 32)
