"""GPU decode parity against the reference (golden fixtures made by the
reference's own CPU path): greedy token IDs identical, logits within 1e-2
relative (norm-relative: max|a-b| / max|b|), int8 KV rows within one step."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err
from tests.golden.fingerprint import gguf_fingerprint

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-2


def _run(name: str, flags: int = 0):
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g["fingerprint"].tobytes()
    m = runtime.CudaModel(path, int(g["ctx"]), flags=flags)
    prompt = [int(t) for t in g["prompt"]]
    steps = len(g["ids"])
    logits = {}
    buf = np.empty(m.vocab, np.float32)
    ids = [m.prefill(prompt, 0, logits=buf)]
    logits[0] = buf.copy()
    pos = len(prompt)
    for s in range(1, steps):
        ids.append(m.forward(ids[-1], pos, logits=buf))
        logits[s] = buf.copy()
        pos += 1
    return g, m, ids, logits


NEAR_TIE = 5e-3  # reference top-1/top-2 margin, as a fraction of max |logit|

# The int8 KV cache rounds every K/V value with roundf (layer_scheduler.c:116),
# so a last-bit difference anywhere upstream can move a value across a .5
# boundary; summing the reference's own fp32 dot products in another order
# already moves its logits by up to ~2e-3 of max |logit| (measured on the
# TinyLlama shape).  A greedy choice whose reference margin is below NEAR_TIE is
# therefore not determined by the reference's arithmetic alone.

FIXTURES = ["tiny", "tiny-mha", "tiny-q8", "tinyllama", "llama2-7b"]


def _near_ties(g) -> np.ndarray:
    tv, am = g["topk_vals"], g["absmax"]
    return (tv[:, 0] - tv[:, 1]) / am < NEAR_TIE


@pytest.mark.parametrize("name", FIXTURES)
def test_greedy_parity(name):
    """Free-running greedy decode: identical to the reference's token IDs for
    every step; a divergence is only accepted at a reference near-tie, and then
    the GPU's choice must be the reference's runner-up."""
    g, m, ids, logits = _run(name)
    ref = [int(t) for t in g["ids"]]
    for i, s in enumerate(g["logit_steps"]):
        if ids[:int(s) + 1] == ref[:int(s) + 1]:
            assert rel_err(logits[int(s)], g["logits"][i]) < LOGIT_RTOL, f"step {s}"
    if ids != ref:
        first = next(i for i, (a, b) in enumerate(zip(ids, ref)) if a != b)
        assert _near_ties(g)[first], f"diverged at step {first} without a near-tie"
        assert ids[first] == int(g["topk_ids"][first][1])
    m.close()


@pytest.mark.parametrize("name", FIXTURES)
def test_teacher_forced_parity(name):
    """Every step fed the reference's own token: the GPU logits at the
    reference's top-4 tokens agree within 1e-2 of max |logit|, and the GPU's
    argmax equals the reference's at every step that is not a near-tie (at a
    near-tie it is one of the reference's top two)."""
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    ref = [int(t) for t in g["ids"]]
    ties = _near_ties(g)
    with runtime.CudaModel(path, int(g["ctx"])) as m:
        buf = np.empty(m.vocab, np.float32)
        prompt = [int(t) for t in g["prompt"]]
        got = m.prefill(prompt, 0, logits=buf)
        # int8 K/V row written by the prompt: within one quantisation step
        k, v, ks, vs = m.kv_row(int(g["kv_layer"]), int(g["kv_pos"]))
        assert np.abs(k.astype(int) - g["k_row"]).max() <= 1
        assert np.abs(v.astype(int) - g["v_row"]).max() <= 1
        assert (k == g["k_row"]).mean() > 0.98 and (v == g["v_row"]).mean() > 0.98
        np.testing.assert_allclose([ks, vs], g["kv_scales"], rtol=1e-3)
        for s in range(len(ref)):
            if s > 0:
                got = m.forward(ref[s - 1], len(prompt) + s - 1, logits=buf)
            top, vals, am = g["topk_ids"][s], g["topk_vals"][s], float(g["absmax"][s])
            assert np.abs(buf[top] - vals).max() / am < LOGIT_RTOL, f"step {s}"
            if ties[s]:
                assert got in (int(top[0]), int(top[1])), f"step {s}"
            else:
                assert got == ref[s], f"step {s}"


@pytest.mark.parametrize("name", ["tiny", "tinyllama"])
def test_device_loop_equals_host_loop(name):
    """ss_cuda_decode_greedy (tokens fed back on the device, one CUDA graph per
    step) produces the same tokens as step-by-step ss_cuda_forward."""
    g, m, ids, _ = _run(name)
    m.reset()
    prompt = [int(t) for t in g["prompt"]]
    first = m.prefill(prompt, 0)
    dev = [first] + m.decode_greedy(first, len(prompt), len(ids) - 1)
    assert dev == ids
    m.close()


def test_no_pdl_no_graph_same_result():
    """PDL/graph chaining changes scheduling only, never results."""
    _, m1, ids1, lg1 = _run("tiny")
    _, m2, ids2, lg2 = _run("tiny", flags=runtime.FLAG_NO_PDL | runtime.FLAG_NO_GRAPH)
    assert ids1 == ids2
    for s in lg1:
        np.testing.assert_array_equal(lg1[s], lg2[s])
    m1.close()
    m2.close()


def test_scheduler_twins_match_reference_oracle():
    """ss_cuda_scheduler_prefill/forward return logits like the reference's
    ss_scheduler_prefill/forward (valid until the next call)."""
    cfg = configs.get("tiny-mha")
    path = synth.ensure_gguf(cfg)
    ref = oracle.OracleModel(path, cfg.ctx)
    prompt = synth.prompt_tokens(cfg)
    with runtime.CudaModel(path, cfg.ctx) as m:
        a = m.scheduler_prefill(prompt, 0)
        b = ref.prefill(prompt, 0)
        assert rel_err(a, b) < 1e-3
        for i in range(4):
            tok = int(np.argmax(b))
            a = m.scheduler_forward(tok, len(prompt) + i)
            b = ref.forward(tok, len(prompt) + i)
            assert rel_err(a, b) < 1e-3
        first = m.scheduler_prefill(prompt, 0)  # KV rows of the prompt rewritten in place
        m.reset()
        np.testing.assert_array_equal(m.scheduler_prefill(prompt, 0), first)


def test_argument_errors():
    cfg = configs.get("tiny")
    with runtime.CudaModel(synth.ensure_gguf(cfg), 16) as m:
        with pytest.raises(runtime.SSCudaError) as e:
            m.forward(1, 16)
        assert e.value.code == -5
        with pytest.raises(runtime.SSCudaError):
            m.forward(cfg.vocab, 0)
        with pytest.raises(runtime.SSCudaError):
            m.decode_greedy(1, 10, 10)
        m.forward(1, 0)  # context still usable
        m.cancel()
        with pytest.raises(runtime.SSCudaError) as e:
            m.decode_greedy(1, 1, 2)
        assert e.value.code == -6
        m.reset()
        m.forward(1, 0)


def test_bad_gguf_rejected(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\xff" * 64)
    with pytest.raises(runtime.SSCudaError):
        runtime.CudaModel(str(bad))
    with pytest.raises(runtime.SSCudaError):
        runtime.CudaModel(str(tmp_path / "missing.gguf"))


def test_deterministic_across_runs():
    _, m1, ids1, lg1 = _run("tiny-q8")
    _, m2, ids2, lg2 = _run("tiny-q8")
    assert ids1 == ids2
    for s in lg1:
        np.testing.assert_array_equal(lg1[s], lg2[s])
