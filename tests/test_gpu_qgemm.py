"""GPU: the many-token tensor-core product (tcgen05, qgemm.cuh) through the C
ABI (ss_cuda_matmul_batch) against the reference's dequant-matvec
(SlipStream/src/core/quantize.c:446-494, via the oracle restatement that is
pinned bit for bit to it) applied to each token on its own.

The product sums in another order than the reference (exact integer block
dot products of 23-bit block fixed-point activations, fp32 across blocks), so
the bar is fp32 rounding: max |gpu - ref| below 2e-6 of the row norm bound
sum_j |w_j x_j| (the error scale of any fp32 evaluation), and far below the
1e-2 logit bar."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.golden.crafted import tensor_table

pytestmark = pytest.mark.gpu

F32P = ctypes.POINTER(ctypes.c_float)
BLOCK = {2: 18, 8: 34}


def _dequant(path, name):
    off, t, dims = tensor_table(path)[name]
    cols, rows = int(dims[0]), int(dims[1])
    raw = np.fromfile(path, np.uint8, count=rows * cols // 32 * BLOCK[t], offset=off)
    w = np.empty(rows * cols, np.float32)
    oracle.oracle_ops().sso_dequantize(raw.ctypes.data, w.ctypes.data_as(F32P), rows * cols, t)
    return raw, t, rows, cols, w.reshape(rows, cols)


def _ref_matvec(raw, t, rows, cols, x):
    out = np.empty(rows, np.float32)
    xx = np.ascontiguousarray(x, np.float32)
    oracle.oracle_ops().sso_dequant_matvec(out.ctypes.data_as(F32P), raw.ctypes.data,
                                          xx.ctypes.data_as(F32P), rows, cols, t)
    return out


NAMES = ["blk.0.attn_q.weight", "blk.0.attn_k.weight", "blk.0.attn_v.weight",
         "blk.0.attn_output.weight", "blk.1.ffn_gate.weight", "blk.1.ffn_up.weight",
         "blk.1.ffn_down.weight", "output.weight"]


@pytest.mark.parametrize("name", ["tiny", "tiny-q8", "tinyllama"])
def test_matmul_batch_matches_reference(name):
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    rng = np.random.default_rng(99)
    with runtime.CudaModel(path, cfg.ctx) as m:
        assert m.stats()["persistent"] == 1
        for tname in NAMES:
            raw, t, rows, cols, w = _dequant(path, tname)
            for T in (1, 3, 16, 17, 32):
                x = rng.standard_normal((T, cols)).astype(np.float32)
                x[:, :32] *= 1e-3  # a block of small values next to ordinary ones
                got = m.matmul_batch(tname, x, rows)
                for k in range(T):
                    ref = _ref_matvec(raw, t, rows, cols, x[k])
                    bound = np.abs(w) @ np.abs(x[k]) + 1e-30
                    err = float(np.max(np.abs(got[k] - ref) / bound))
                    assert err < 2e-6, f"{tname} T={T} token {k}: {err:.3g}"


def test_matmul_batch_rejects_bad_arguments():
    cfg = configs.get("tiny")
    with runtime.CudaModel(synth.ensure_gguf(cfg), cfg.ctx) as m:
        x = np.zeros((33, cfg.d_model), np.float32)
        with pytest.raises(runtime.SSCudaError):
            m.matmul_batch("blk.0.attn_q.weight", x, cfg.d_model)
        with pytest.raises(runtime.SSCudaError):
            m.matmul_batch("no.such.weight", x[:2], cfg.d_model)
