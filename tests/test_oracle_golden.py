"""The CPU oracle restatement (oracle/ss_oracle.c) against the golden fixtures
made by the reference's own C code (tests/golden/make_golden.py).  The
restatement follows the reference's arithmetic order, so greedy IDs and the
recorded logits must be bit-identical."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, synth
from tests.conftest import load_golden
from tests.golden.fingerprint import gguf_fingerprint

SMALL = ["tiny", "tiny-mha", "tiny-q8"]


@pytest.mark.parametrize("name", SMALL + ["tinyllama"])
def test_greedy_and_logits_bitexact(name):
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g["fingerprint"].tobytes(), "synthetic GGUF bytes changed"
    m = oracle.OracleModel(path, int(g["ctx"]), cap512=True)
    steps = len(g["ids"])
    assert [int(t) for t in g["prompt"]] == synth.prompt_tokens(cfg)
    ids, kept = m.greedy(g["prompt"], steps, keep_logits=set(int(s) for s in g["logit_steps"]))
    assert ids == [int(t) for t in g["ids"]]
    for i, s in enumerate(g["logit_steps"]):
        np.testing.assert_array_equal(kept[int(s)], g["logits"][i])
    k, v, ks, vs = m.kv_row(int(g["kv_layer"]), int(g["kv_pos"]))
    np.testing.assert_array_equal(k, g["k_row"])
    np.testing.assert_array_equal(v, g["v_row"])
    np.testing.assert_array_equal(np.array([ks, vs], np.float32), g["kv_scales"])


def test_prefill_equals_token_by_token():
    """Layer-major prefill (layer_scheduler.c:720-743) == per-token forward."""
    cfg = configs.get("tiny")
    path = synth.ensure_gguf(cfg)
    a = oracle.OracleModel(path, cfg.ctx)
    b = oracle.OracleModel(path, cfg.ctx)
    prompt = synth.prompt_tokens(cfg)
    la = a.prefill(prompt)
    for i, t in enumerate(prompt):
        lb = b.forward(t, i)
    np.testing.assert_array_equal(la, lb)


def test_reset_clears_state():
    cfg = configs.get("tiny")
    m = oracle.OracleModel(synth.ensure_gguf(cfg), cfg.ctx)
    prompt = synth.prompt_tokens(cfg)
    first = m.prefill(prompt)
    m.forward(3, len(prompt))
    m.reset()
    np.testing.assert_array_equal(m.prefill(prompt), first)


def test_position_bounds_rejected():
    cfg = configs.get("tiny")
    m = oracle.OracleModel(synth.ensure_gguf(cfg), 16, cap512=True)
    with pytest.raises(RuntimeError):
        m.forward(1, 16)
    with pytest.raises(RuntimeError):
        m.forward(cfg.vocab, 0)


def test_noise_floor_fixture_matches_oracle():
    """tests/golden/noise_floor.json (the tolerance source of the GPU parity
    tests) is reproduced by the oracle's blocked summation order."""
    import json
    import os
    from tests.golden.noise_floor import measure
    path = os.path.join(os.path.dirname(__file__), "golden", "noise_floor.json")
    rec = json.load(open(path))["tiny"]
    got = measure("tiny", rec["steps"])
    assert abs(got["max_step_inf_rel"] - rec["max_step_inf_rel"]) <= 1e-9
    assert got["prefill_inf_rel"] > 0.0  # the two orders do differ


@pytest.mark.parametrize("name", SMALL + ["tinyllama"])
def test_embed_bitexact(name):
    """The restatement's sentence embedding (sso_embed) against the reference's
    ss_scheduler_embed vectors in embed.npz: bit-identical."""
    g = load_golden("embed")
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g[f"{name}_fingerprint"].tobytes()
    for key in ("prompt", "one", "long"):
        if f"{name}_{key}_tokens" not in g:
            continue
        m = oracle.OracleModel(path, cfg.ctx, cap512=True)
        np.testing.assert_array_equal(m.embed(g[f"{name}_{key}_tokens"]), g[f"{name}_{key}_embed"])
        m.close()
