"""Several sequences decoded together (ss_cuda_forward with n_seq > 1,
ss_cuda_prefill_batch): each sequence's logits and greedy tokens against the
reference's path for that sequence alone.

* small configurations: every sequence against this repository's C
  restatement of the reference (oracle/ss_oracle.c, the reference's order),
  teacher-forced on the restatement's tokens;
* the full-size configurations the batched decode is quoted on (Llama-3-8B
  Q8_0 at B = 8, the 70B shape at B = 16): sequence 0 carries the golden
  fixture's prompt and must reproduce the reference's own tokens and logits
  (tests/golden, made by the reference's CPU path), the other sequences
  carry other prompts;
* size-independent properties: a sequence's results do not depend on which
  other sequences share its batch (bitwise), and the context keeps decoding
  sequence 0 on its own afterwards.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err
from tests.golden.fingerprint import gguf_fingerprint
from tests.test_gpu_decode import _acceptable_choice, logit_tol, report

pytestmark = pytest.mark.gpu


def _prompts(cfg, g, n_seq: int, length: int) -> np.ndarray:
    """n_seq prompts of `length` tokens: row 0 the fixture's prompt (when a
    fixture is given), the others seeded uniform token IDs."""
    rng = np.random.default_rng(1234)
    p = rng.integers(0, cfg.vocab, size=(n_seq, length), dtype=np.int64).astype(np.int32)
    if g is not None:
        p[0] = np.asarray(g["prompt"], np.int32)[:length]
    return p


@pytest.mark.parametrize("name", ["tiny", "tiny-q8", "tinyllama"])
def test_batched_decode_matches_oracle(name):
    """B = 4 sequences with different prompts, teacher-forced on the
    restatement's greedy tokens: every sequence's logits within the
    configuration's tolerance at every step, and its greedy token the
    restatement's wherever the restatement's margin exceeds the tolerance."""
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    tol = logit_tol(name)
    g = load_golden(name)
    n_seq, steps = 4, 12
    prompts = _prompts(cfg, g, n_seq, len(g["prompt"]))
    ref = oracle.OracleModel(path, cfg.ctx)
    want_ids, want_logits = [], []
    for s in range(n_seq):
        ref.reset()
        ids, lg = ref.greedy(prompts[s].tolist(), steps, keep_logits=range(steps))
        want_ids.append(ids)
        want_logits.append(lg)
    ref.close()
    n = prompts.shape[1]
    with runtime.CudaModel(path, cfg.ctx, max_batch=n_seq) as m:
        assert m.max_batch == n_seq
        logits = np.empty((n_seq, m.vocab), np.float32)
        got = m.prefill_batch(prompts, 0, logits=logits)
        worst = 0.0
        for step in range(steps):
            if step > 0:
                toks = [want_ids[s][step - 1] for s in range(n_seq)]
                got = m.forward_batch(toks, n + step - 1, logits=logits)
            for s in range(n_seq):
                e = rel_err(logits[s], want_logits[s][step])
                worst = max(worst, e)
                assert e < tol, f"sequence {s} step {step}: {e}"
                top2 = np.sort(want_logits[s][step])[-2:]
                margin = float(top2[1] - top2[0]) / float(np.abs(want_logits[s][step]).max())
                if margin > tol:
                    assert got[s] == want_ids[s][step], f"sequence {s} step {step}"
        report(name, "batched", mode="teacher-forced vs restatement", n_seq=n_seq, steps=steps,
               max_rel_logit_err=worst, tol=tol)


@pytest.mark.parametrize("name", ["tiny-q8", "tinyllama"])
def test_sequence_independent_of_batch(name):
    """A sequence's logits are bitwise the same whether it decodes among 4 or
    among 2 sequences (the product keeps every token's column separate)."""
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    g = load_golden(name)
    prompts = _prompts(cfg, g, 4, len(g["prompt"]))
    n = prompts.shape[1]
    out = {}
    for B in (4, 2):
        with runtime.CudaModel(path, cfg.ctx, max_batch=4) as m:
            lg = np.empty((B, m.vocab), np.float32)
            toks = m.prefill_batch(prompts[:B], 0, logits=lg)
            rows = [lg[:2].copy()]
            for step in range(3):
                toks = m.forward_batch(toks, n + step, logits=lg)
                rows.append(lg[:2].copy())
            out[B] = rows
    for a, b in zip(out[4], out[2]):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("name,n_seq", [("llama3-8b", 8), ("llama2-70b-4l", 16)])
def test_batched_full_size_against_reference(name, n_seq):
    """The configurations the batched decode is quoted on: B sequences, sequence
    0 with the golden fixture's prompt.  Sequence 0 reproduces the reference's
    greedy tokens (a divergence only where the reference's own top-2 lie within
    the tolerance) with logits within the tolerance at the recorded steps; every
    sequence's logits are finite."""
    g = load_golden(name)
    cfg = configs.get(str(g["config"]))
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g["fingerprint"].tobytes()
    tol = logit_tol(name)
    ref = [int(t) for t in g["ids"]]
    prompts = _prompts(cfg, g, n_seq, len(g["prompt"]))
    n = prompts.shape[1]
    with runtime.CudaModel(path, int(g["ctx"]), max_batch=n_seq) as m:
        lg = np.empty((n_seq, m.vocab), np.float32)
        toks = m.prefill_batch(prompts, 0, logits=lg)
        ids, logits = [toks[0]], {0: lg[0].copy()}
        assert np.isfinite(lg).all()
        for step in range(1, len(ref)):
            toks = m.forward_batch(toks, n + step - 1, logits=lg)
            ids.append(toks[0])
            logits[step] = lg[0].copy()
            assert np.isfinite(lg).all()
    first = next((i for i, (a, b) in enumerate(zip(ids, ref)) if a != b), len(ref))
    errs = {int(s): rel_err(logits[int(s)], g["logits"][i])
            for i, s in enumerate(g["logit_steps"]) if int(s) <= first}
    report(name, f"batched B={n_seq}", mode="free-running", steps=len(ref), first_divergence=first,
           identical_ids=first == len(ref), max_rel_logit_err=max(errs.values()), tol=tol)
    for s, e in errs.items():
        assert e < tol, f"step {s}"
    if first < len(ref):
        assert _acceptable_choice(g, first, ids[first], tol), f"diverged at step {first}"


def test_single_sequence_continues_after_batch():
    """After a batched prompt and batched steps, sequence 0 decodes on its own
    (the persistent step) from its cache: the fixture's greedy tokens."""
    name = "tinyllama"
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    ref = [int(t) for t in g["ids"]]
    prompts = _prompts(cfg, g, 3, len(g["prompt"]))
    n = prompts.shape[1]
    with runtime.CudaModel(path, int(g["ctx"]), max_batch=3) as m:
        assert m.stats()["persistent"] == 1
        toks = m.prefill_batch(prompts, 0)
        ids = [toks[0]]
        for step in range(1, 4):
            toks = m.forward_batch(toks, n + step - 1)
            ids.append(toks[0])
        ids += m.decode_greedy(ids[-1], n + 3, 12)
    assert ids == ref[:16]


def test_many_token_step_without_persistent_step():
    """A context that decodes several sequences but runs no persistent step
    (forced here with SS_CUDA_FLAG_MULTI_KERNEL; on one GPU the 70B shape gets
    there by itself) takes every single-sequence step through the many-token
    kernels, with the token and position read on the device: prefill, the
    device greedy loop and the host loop give the fixture's tokens."""
    name = "tinyllama"
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    ref = [int(t) for t in g["ids"]]
    tol = logit_tol(name)
    prompt = [int(t) for t in g["prompt"]]
    with runtime.CudaModel(path, int(g["ctx"]), flags=runtime.FLAG_MULTI_KERNEL, max_batch=2) as m:
        st = m.stats()
        assert st["persistent"] == 0
        first = m.prefill(prompt, 0)
        ids = [first] + m.decode_greedy(first, len(prompt), 15)
        m.reset()
        buf = np.empty(m.vocab, np.float32)
        host = [m.prefill(prompt, 0)]
        for s in range(1, 16):
            host.append(m.forward(host[-1], len(prompt) + s - 1, logits=buf))
            if s in [int(v) for v in g["logit_steps"]]:
                i = [int(v) for v in g["logit_steps"]].index(s)
                assert rel_err(buf, g["logits"][i]) < tol
    assert ids == host
    first_div = next((i for i, (a, b) in enumerate(zip(ids, ref)) if a != b), 16)
    if first_div < 16:
        assert _acceptable_choice(g, first_div, ids[first_div], tol)


def test_batch_argument_errors():
    cfg = configs.get("tiny")
    path = synth.ensure_gguf(cfg)
    with pytest.raises(runtime.SSCudaError):
        runtime.CudaModel(path, cfg.ctx, max_batch=33)
    with runtime.CudaModel(path, cfg.ctx) as m:  # one sequence
        with pytest.raises(runtime.SSCudaError):
            m.forward_batch([1, 2], 0)
        with pytest.raises(runtime.SSCudaError):
            m.prefill_batch(np.ones((2, 4), np.int32), 0)
        m.forward(1, 0)
    with runtime.CudaModel(path, cfg.ctx, max_batch=2) as m:
        with pytest.raises(runtime.SSCudaError):
            m.forward_batch([1, 2, 3], 0)  # above max_batch
        with pytest.raises(runtime.SSCudaError):
            m.forward_batch([1, cfg.vocab], 0)  # token outside the vocabulary
        with pytest.raises(runtime.SSCudaError):
            m.forward_batch([1, 2], cfg.ctx)  # position outside the context
        assert m.forward_batch([1, 2], 0) == m.forward_batch([1, 2], 0)
