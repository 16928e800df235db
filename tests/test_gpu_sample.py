"""Sampling on the device (ss_cuda_sample_logits / ss_cuda_sample /
ss_cuda_decode_sample) against ss_sample (SlipStream/src/core/tensor.c:
363-451):

* every case of tests/golden/sample_cases.py, DRAWS chained draws: the token
  and RNG state of the restatement with the GPU's exponential (bit-exact by
  construction -- the same sums in the same order), and the reference's own
  draws from the golden fixture (equal except where libm's expf rounds a last
  bit differently and that moves a running sum across a threshold; counted and
  reported, and each such draw must be the restatement's);
* the generation loop on the device (engine.c:233-289): its tokens equal a host
  replay that draws with the restatement from the same context's logits step
  by step, on the persistent step and on the many-token step;
* several sequences sampled together (ss_cuda_decode_sample_batch) against a
  host replay of the same batched steps;
* temperature <= 0 is the greedy argmax and leaves the RNG state alone.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden
from tests.golden import sample_cases as sc
from tests.test_gpu_decode import report

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    with runtime.CudaModel(None) as m:  # no model: the op-level entry point only
        yield m


def test_sample_logits_matches_reference(ctx):
    g = load_golden("sample")
    differ, total = 0, 0
    for name, (make, *_rest) in sc.CASES.items():
        assert g[f"{name}/digest"].tobytes() == sc.digest(make()), name
        got_t, got_s = sc.draws(lambda x, t, p, k, s: ctx.sample_logits(x, t, p, k, s), name)
        dd_t, dd_s = sc.draws(lambda x, t, p, k, s: oracle.sample(x, t, p, k, s, 1), name)
        assert got_t == dd_t and got_s == dd_s, name
        want = [int(v) for v in g[f"{name}/tokens"]]
        assert got_s == [int(v) for v in g[f"{name}/states"]], name
        differ += sum(a != b for a, b in zip(got_t, want))
        total += len(want)
    report("sample", "ss_cuda_sample_logits", cases=len(sc.CASES), draws=total,
           draws_differing_from_reference=differ)
    assert differ <= total // 100


def test_sample_argument_errors(ctx):
    x = np.zeros(10, np.float32)
    lib = runtime.load_library()
    tok = runtime.ctypes.c_int32()
    # sampling needs an RNG state; greedy does not
    assert lib.ss_cuda_sample_logits(ctx._h, runtime._f(x), 10, 1.0, 1.0, 0, None,
                                     runtime.ctypes.byref(tok)) == -5
    assert lib.ss_cuda_sample_logits(ctx._h, runtime._f(x), 10, 0.0, 1.0, 0, None,
                                     runtime.ctypes.byref(tok)) == 0
    assert tok.value == 0
    with pytest.raises(runtime.SSCudaError):
        ctx.sample_logits(np.zeros(0, np.float32), 1.0, 1.0, 0, 1)
    with pytest.raises(runtime.SSCudaError):
        ctx.sample(1.0, 1.0, 0, 1)  # no model, no logits


def _replay(m, cfg, prompt, n, t, p, k, state):
    """engine.c's loop on the host: draw with the restatement (the GPU's
    exponential) from this context's logits, forward the token, repeat."""
    m.reset()
    lg = np.empty(m.vocab, np.float32)
    m.prefill(prompt, 0, logits=lg)
    ids, s = [], state
    for i in range(n):
        tok, s = oracle.sample(lg, t, p, k, s, 1)
        ids.append(tok)
        if i + 1 < n:
            m.forward(tok, len(prompt) + i, logits=lg)
    return ids, s


@pytest.mark.parametrize("name,flags,max_batch", [("tinyllama", 0, 1), ("tiny-q8", 0, 1),
                                                  ("tinyllama", runtime.FLAG_MULTI_KERNEL, 2)])
def test_decode_sample_matches_host_replay(name, flags, max_batch):
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    prompt = synth.prompt_tokens(cfg)
    n = 24
    settings = [(0.8, 0.95, 40, 0x9E3779B97F4A7C15), (1.0, 0.9, 0, 0xD1B54A32D192ED03),
                (1.5, 1.0, 0, 0x2545F4914F6CDD1D)]
    with runtime.CudaModel(path, cfg.ctx, flags=flags, max_batch=max_batch) as m:
        if flags:
            assert m.stats()["persistent"] == 0
        for t, p, k, seed in settings:
            m.reset()
            m.prefill(prompt, 0)
            ids, state = m.decode_sample(len(prompt), n, t, p, k, seed)
            want, want_state = _replay(m, cfg, prompt, n, t, p, k, seed)
            assert ids == want, (t, p, k)
            assert state == want_state
            # ss_cuda_sample draws from the logits on the device the same way
            m.reset()
            lg = np.empty(m.vocab, np.float32)
            m.prefill(prompt, 0, logits=lg)
            assert m.sample(t, p, k, seed) == oracle.sample(lg, t, p, k, seed, 1)
        report(name, "decode_sample", flags=flags, tokens=n, settings=len(settings), identical=True)


def test_decode_sample_greedy_is_decode_greedy():
    name = "tinyllama"
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    g = load_golden(name)
    prompt = [int(v) for v in g["prompt"]]
    with runtime.CudaModel(path, cfg.ctx) as m:
        m.prefill(prompt, 0)
        ids, state = m.decode_sample(len(prompt), 16, 0.0, 0.9, 40, 777)
        assert state == 777
        m.reset()
        first = m.prefill(prompt, 0)
        assert ids == [first] + m.decode_greedy(first, len(prompt), 15)
        # the position is the last draw's: ss_cuda_decode_steps continues from it
        m.reset()
        m.prefill(prompt, 0)
        ids2, _ = m.decode_sample(len(prompt), 8, 0.0, 1.0, 0, 0)
        m.decode_steps(8)
        assert ids2 + m.decode_read(len(prompt) + 8, 8) == ids


def test_decode_sample_argument_errors():
    cfg = configs.get("tiny")
    path = synth.ensure_gguf(cfg)
    with runtime.CudaModel(path, cfg.ctx) as m:
        m.prefill([1, 2, 3], 0)
        with pytest.raises(runtime.SSCudaError):
            m.decode_sample(3, cfg.ctx, 1.0, 1.0, 0, 1)  # past the context
        with pytest.raises(runtime.SSCudaError):
            m.decode_sample(3, 0, 1.0, 1.0, 0, 1)
        ids, _ = m.decode_sample(cfg.ctx, 1, 1.0, 1.0, 0, 5)  # one draw into the last slot
        assert 0 <= ids[0] < cfg.vocab


@pytest.mark.parametrize("name", ["llama2-7b", "llama3-8b"])
def test_sampler_time(name):
    """Device time of one draw over the configuration's vocabulary (32,000 /
    128,256 logits), reported beside the decode step."""
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    with runtime.CudaModel(path, cfg.ctx) as m:
        m.prefill(synth.prompt_tokens(cfg, 8), 0)
        typical = m.time_kernel("sample", 20)
        longest = m.time_kernel("sample_topp", 20)
    report(name, "sampler", vocab=cfg.vocab, ms_typical=typical, ms_top_p_only=longest)
    assert typical > 0 and longest > 0


@pytest.mark.parametrize("name", ["tinyllama", "tiny-q8"])
def test_decode_sample_batch_matches_host_replay(name):
    """Several sequences sampled together (ss_cuda_decode_sample_batch): every
    sequence's tokens and RNG state equal a host replay that steps the same
    sequences with host logits (ss_cuda_forward, n_seq > 1) and draws each row
    with the restatement; temperature 0 is the greedy batched loop."""
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    n_seq, steps, plen = 4, 12, 8
    rng = np.random.default_rng(77)
    prompts = rng.integers(0, cfg.vocab, size=(n_seq, plen)).astype(np.int32)
    states0 = [int(v) for v in rng.integers(1, 2**62, size=n_seq, dtype=np.int64)]
    with runtime.CudaModel(path, cfg.ctx, max_batch=n_seq) as m:
        for t, p, k in [(0.7, 0.9, 40), (1.0, 0.95, 0), (1.3, 1.0, 0)]:
            m.reset()
            first = m.prefill_batch(prompts, 0)
            ids, states = m.decode_sample_batch(first, plen, steps, t, p, k, states0)
            m.reset()
            toks = m.prefill_batch(prompts, 0)
            lg = np.empty((n_seq, m.vocab), np.float32)
            st, want = list(states0), []
            for step in range(steps):
                m.forward_batch(toks, plen + step, logits=lg)
                nxt = []
                for s in range(n_seq):
                    tok, st[s] = oracle.sample(lg[s], t, p, k, st[s], 1)
                    nxt.append(tok)
                want.append(nxt)
                toks = nxt
            assert ids.tolist() == want, (t, p, k)
            assert states == st
        m.reset()
        first = m.prefill_batch(prompts, 0)
        ids, states = m.decode_sample_batch(first, plen, steps, 0.0, 0.9, 40, states0)
        assert states == states0
        m.reset()
        first = m.prefill_batch(prompts, 0)
        assert ids.tolist() == m.decode_greedy_batch(first, plen, steps).tolist()
        with pytest.raises(runtime.SSCudaError):
            m.decode_sample_batch([1] * (n_seq + 1), plen, 2, 1.0, 1.0, 0, [1] * (n_seq + 1))
    report(name, "decode_sample_batch", n_seq=n_seq, steps=steps, settings=3, identical=True)
