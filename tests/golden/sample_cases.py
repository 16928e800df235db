"""Inputs of the sampling parity cases -- TEST INFRASTRUCTURE.

ss_sample (SlipStream/src/core/tensor.c:363-451) is checked on logits vectors
built here from a seed (the fixture records a digest of each vector, so a
change in numpy's generators shows up as a digest mismatch rather than as a
parity failure): seeded normal logits at several vocabulary sizes and spreads,
and crafted edge cases -- NaN and infinite logits, all-equal logits, ties at
the top-k boundary, probabilities in the float subnormal range, and the
greedy, tiny- and huge-temperature settings.

``CASES`` maps a case name to (logits builder, temperature, top_p, top_k,
initial RNG state); each case is drawn ``DRAWS`` times in a row, the RNG state
carried from draw to draw as ss_generate carries it (engine.c:202, 242-244).
Used by tests/golden/make_golden.py (expectations from the reference build),
tests/test_oracle_sample.py and tests/test_gpu_sample.py.
"""
from __future__ import annotations

import hashlib

import numpy as np

DRAWS = 8


def _normal(n: int, scale: float, seed: int):
    def make() -> np.ndarray:
        return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)
    return make


def _crafted(kind: str, n: int, seed: int):
    def make() -> np.ndarray:
        rng = np.random.default_rng(seed)
        x = rng.standard_normal(n).astype(np.float32)
        if kind == "nan":  # NaN logits, index 0 among them (read as -FLT_MAX)
            x[rng.integers(0, n, size=max(1, n // 50))] = np.nan
            x[0] = np.nan
        elif kind == "posinf":  # one +inf: every probability becomes NaN
            x[n // 3] = np.inf
        elif kind == "neginf":  # -inf logits have probability 0
            x[rng.integers(0, n, size=max(1, n // 4))] = -np.inf
        elif kind == "equal":  # a uniform distribution: ties everywhere in the sort
            x[:] = np.float32(0.25)
        elif kind == "ties":  # the 10 largest values appear twice each
            top = np.sort(x)[-10:]
            x[rng.integers(0, n, size=10)] = top
        elif kind == "subnormal":  # exp(x - max) down into the float subnormal range
            x = rng.uniform(-104.0, 0.0, size=n).astype(np.float32)
        elif kind == "peaked":  # most probabilities underflow to 0
            x = (x * 60.0).astype(np.float32)
        elif kind == "allnan":
            x[:] = np.nan
        return x
    return make


_SEEDS = [0x9E3779B97F4A7C15, 0xD1B54A32D192ED03, 0x2545F4914F6CDD1D, 0x1, 0xFFFFFFFFFFFFFFFF,
          0x0123456789ABCDEF, 0x7FFFFFFFFFFFFFFF, 0x5DEECE66D]

CASES: dict = {}


def _add(name, make, temperature, top_p, top_k, seed_index):
    CASES[name] = (make, float(temperature), float(top_p), int(top_k), _SEEDS[seed_index % len(_SEEDS)])


# seeded normal logits (vocabulary sizes of the configurations included)
_PARAMS = [(1.0, 1.0, 0), (0.8, 0.95, 40), (0.7, 0.9, 0), (1.2, 1.0, 50), (0.5, 0.5, 0),
           (1.0, 0.999, 0), (2.0, 0.9, 5), (1.0, 1e-6, 0), (1.0, 0.9, 1), (0.0, 0.9, 40),
           (-1.0, 1.0, 0), (1e-4, 1.0, 0), (100.0, 0.9, 0), (0.9, 0.8, 300)]
_i = 0
for n in (1, 2, 3, 17, 100, 1000, 5003, 32000, 128256):
    for scale in (0.5, 1.3, 4.0):
        t, p, k = _PARAMS[_i % len(_PARAMS)]
        _add(f"normal-n{n}-s{scale}-{_i}", _normal(n, scale, 1000 + _i), t, p, k, _i)
        _i += 1
for t, p, k in _PARAMS:  # every setting on the 32000-logit shape
    _add(f"normal-n32000-T{t}-p{p}-k{k}", _normal(32000, 1.3, 5000 + _i), t, p, k, _i)
    _i += 1
# edge cases
for kind in ("nan", "posinf", "neginf", "equal", "ties", "subnormal", "peaked", "allnan"):
    for n, (t, p, k) in ((1000, (0.8, 0.9, 40)), (32000, (1.0, 0.95, 0)), (257, (1.0, 1.0, 10))):
        _add(f"{kind}-n{n}-T{t}-p{p}-k{k}", _crafted(kind, n, 7000 + _i), t, p, k, _i)
        _i += 1
_add("nan-temperature", _normal(500, 1.0, 9001), float("nan"), 0.9, 10, 2)
_add("topk-equals-n-minus-1", _normal(300, 1.0, 9002), 1.0, 1.0, 299, 3)
_add("topk-above-n", _normal(300, 1.0, 9003), 1.0, 0.9, 1000, 4)


def digest(x: np.ndarray) -> bytes:
    return hashlib.sha256(np.ascontiguousarray(x, np.float32).tobytes()).digest()[:16]


def draws(fn, name: str) -> tuple[list[int], list[int]]:
    """DRAWS chained draws of case `name` with fn(logits, T, top_p, top_k,
    state) -> (token, state): the tokens and the states after each draw."""
    make, t, p, k, s = CASES[name]
    x = make()
    toks, states = [], []
    for _ in range(DRAWS):
        tok, s = fn(x, t, p, k, s)
        toks.append(tok)
        states.append(s)
    return toks, states
