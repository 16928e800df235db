"""Every GGUF block type of SlipStream's ss_dequantize
(SlipStream/src/core/quantize.c:389-442) and its Q4_K dequant-matvec
(:446-494), on the CPU: the oracle's restatement against the reference's own
outputs (tests/golden/quant.npz), bit for bit."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from tests.conftest import load_golden
from tests.golden import quant_cases as qc

F32P = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def golden():
    return load_golden("quant")


@pytest.mark.parametrize("t", sorted(qc.TYPES), ids=[qc.NAMES[t] for t in sorted(qc.TYPES)])
def test_oracle_dequantize_bitexact(golden, t):
    raw, n = qc.blocks(t)
    np.testing.assert_array_equal(raw, golden[f"{qc.NAMES[t]}/blocks"])
    out = np.empty(n, np.float32)
    oracle.oracle_ops().sso_dequantize(raw.ctypes.data, out.ctypes.data_as(F32P), n, t)
    np.testing.assert_array_equal(out.view(np.uint32), golden[f"{qc.NAMES[t]}/values"].view(np.uint32))


def test_oracle_q4k_matvec_bitexact(golden):
    raw, x = qc.q4k_matrix()
    out = np.empty(48, np.float32)
    oracle.oracle_ops().sso_dequant_matvec(out.ctypes.data_as(F32P), raw.ctypes.data, x.ctypes.data_as(F32P),
                                           48, 1024, 12)
    np.testing.assert_array_equal(out.view(np.uint32), golden["q4k_mv/out"].view(np.uint32))
