"""Single ops of the oracle restatement against the reference's known answers:
the f16->f32 cases of SlipStream/tests/test_quantize.c:33-50, the fp32
matvec/softmax/argmax cases of SlipStream/tests/test_tensor_ops.c:71-118, and
the seeded op vectors the reference produced (tests/golden/ops.npz)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from tests.conftest import load_golden

F32P = ctypes.POINTER(ctypes.c_float)


def fp(a):
    return a.ctypes.data_as(F32P)


@pytest.fixture(scope="module")
def ops():
    return oracle.oracle_ops()


def test_f16_known_answers(ops):
    for h, want in ((0x0000, 0.0), (0x3C00, 1.0), (0xBC00, -1.0), (0x3800, 0.5)):
        assert ops.sso_f16_to_f32(h) == want
    g = load_golden("ops")
    got = np.array([ops.sso_f16_to_f32(int(h)) for h in g["f16_in"]], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), g["f16_out"].view(np.uint32))


@pytest.mark.parametrize("kind,t", [("q4_0", 2), ("q8_0", 8)])
def test_dequant_bitexact(ops, kind, t):
    g = load_golden("ops")
    raw, want = g[f"{kind}_raw"], g[f"{kind}_deq"]
    out = np.empty_like(want)
    ops.sso_dequantize(raw.ctypes.data, fp(out), want.size, t)
    np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind,t", [("q4_0", 2), ("q8_0", 8)])
def test_dequant_matvec_bitexact(ops, kind, t):
    g = load_golden("ops")
    raw, x, want = g[f"{kind}_raw"], g[f"{kind}_x"], g[f"{kind}_mv"]
    out = np.empty_like(want)
    ops.sso_dequant_matvec(fp(out), raw.ctypes.data, fp(x), want.size, x.size, t)
    np.testing.assert_array_equal(out, want)


def test_rmsnorm_rope_softmax_argmax(ops):
    g = load_golden("ops")
    out = np.empty_like(g["rms_out"])
    ops.sso_rmsnorm(fp(out), fp(g["rms_x"]), fp(g["rms_w"]), out.size, np.float32(1e-5))
    np.testing.assert_array_equal(out, g["rms_out"])
    for pos, theta in ((0, 10000.0), (7, 10000.0), (383, 10000.0), (1000, 500000.0)):
        q, k = g["rope_q_in"].copy(), g["rope_k_in"].copy()
        ops.sso_rope(fp(q), fp(k), 4, 2, 16, 16, pos, np.float32(theta))
        np.testing.assert_array_equal(q, g[f"rope_q_{pos}"])
        np.testing.assert_array_equal(k, g[f"rope_k_{pos}"])
    s = g["softmax_in"].copy()
    ops.sso_softmax(fp(s), s.size)
    np.testing.assert_array_equal(s, g["softmax_out"])
    x = np.array([1.0, 3.0, 2.0, 5.0, 4.0], np.float32)  # test_tensor_ops.c:116-119
    assert ops.sso_argmax(fp(x), 5) == 3
    ties = g["argmax_ties_in"]
    assert ops.sso_argmax(fp(ties), ties.size) == int(g["argmax_ties_out"]) == 1


def test_kv_encode(ops):
    """kv_turboquant_encode (layer_scheduler.c:101-118): zero vector, exact .5
    ties (roundf rounds half away from zero), saturation at +-127."""
    zero = np.zeros(8, np.float32)
    q = np.empty(8, np.int8)
    sc = np.zeros(1, np.float32)
    ops.sso_kv_encode(fp(zero), q.ctypes.data, fp(sc), 8)
    assert sc[0] == 0.0 and not q.any()
    v = np.array([127.0, -127.0, 0.5, -0.5, 1.5, 63.5, -2.5, 0.0], np.float32)
    ops.sso_kv_encode(fp(v), q.ctypes.data, fp(sc), 8)
    assert sc[0] == np.float32(1.0)
    assert list(q) == [127, -127, 1, -1, 2, 64, -3, 0]


def test_argmax_edge_cases(ops):
    """The restatement's argmax against the reference's on NaN / signed-zero /
    tie / infinity cases (tests/golden/argmax.npz, made by the reference)."""
    from tests.golden import crafted
    g = load_golden("argmax")
    for name, a in crafted.argmax_arrays().items():
        assert ops.sso_argmax(fp(a), a.size) == int(g[f"want_{name}"]), name
        if f"in_{name}" in g:
            np.testing.assert_array_equal(g[f"in_{name}"].view(np.uint32), a.view(np.uint32))
