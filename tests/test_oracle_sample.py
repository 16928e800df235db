"""Sampling (ss_sample, SlipStream/src/core/tensor.c:363-451) on the CPU: the
oracle's restatement against the reference's own draws (tests/golden/
sample.npz, made by the reference build), and the exponential the GPU sampler
uses against a double-precision exp rounded to float."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.conftest import load_golden
from tests.golden import sample_cases as sc


@pytest.fixture(scope="module")
def golden():
    return load_golden("sample")


def test_cases_regenerate_identically(golden):
    for name, (make, *_rest) in sc.CASES.items():
        assert golden[f"{name}/digest"].tobytes() == sc.digest(make()), name


def test_oracle_sample_matches_reference(golden):
    """The restatement with libm's expf (the reference's arithmetic) gives the
    reference's token and RNG state at every draw of every case."""
    for name in sc.CASES:
        toks, states = sc.draws(lambda x, t, p, k, s: oracle.sample(x, t, p, k, s, 0), name)
        assert toks == [int(v) for v in golden[f"{name}/tokens"]], name
        assert states == [int(v) for v in golden[f"{name}/states"]], name


def test_oracle_sample_gpu_exponential(golden):
    """With the GPU sampler's exponential the draws stay the reference's except
    where libm's expf and the correctly rounded value differ in a last bit that
    moves a running sum across a threshold; count those (expected: none or
    very few)."""
    diff = 0
    total = 0
    for name in sc.CASES:
        toks, states = sc.draws(lambda x, t, p, k, s: oracle.sample(x, t, p, k, s, 1), name)
        want = [int(v) for v in golden[f"{name}/tokens"]]
        diff += sum(a != b for a, b in zip(toks, want))
        total += len(want)
        assert states == [int(v) for v in golden[f"{name}/states"]], name  # one RNG step per draw
    print(f"draws differing from the reference with the double-precision exponential: {diff} of {total}")
    assert diff <= total // 100


def test_exp_dd_is_correctly_rounded():
    """sso_exp_dd (the GPU sampler's e^x) against numpy's double exp rounded to
    float: equal on a million seeded arguments over the softmax's range and on
    the special values, including float subnormal results."""
    rng = np.random.default_rng(42)
    x = np.concatenate([
        -rng.random(1_000_000).astype(np.float32) * np.float32(110.0),
        np.array([0.0, -0.0, -1e-30, -1e-8, -0.5, -1.0, -87.3365, -88.0, -103.0, -103.97, -104.0,
                  -150.0, -200.0, -250.0, 1.0, 10.0, 88.7, 88.72, 89.0, 300.0, -np.inf, np.inf],
                 np.float32)])
    got = oracle.exp_dd(x)
    with np.errstate(over="ignore"):
        want = np.exp(x.astype(np.float64)).astype(np.float32)
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size <= 2, [(float(x[i]), float(got[i]), float(want[i])) for i in bad[:5]]
    assert np.isnan(oracle.exp_dd(np.array([np.nan], np.float32)))[0]


def test_greedy_draw_leaves_rng_state():
    x = np.array([0.5, 2.0, 2.0, -1.0], np.float32)
    assert oracle.sample(x, 0.0, 0.9, 40, 12345) == (1, 12345)
    assert oracle.sample(x, -3.0, 1.0, 0, 7) == (1, 7)
