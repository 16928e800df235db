"""Sentence embedding (ss_cuda_embed / ss_cuda_scheduler_embed, the twin of
ss_scheduler_embed, SlipStream/src/core/layer_scheduler.c:805-915) on the GPU
against the reference's own vectors (tests/golden/embed.npz, made by the
reference's CPU path): within the configuration's logit tolerance of max |e|,
unit L2 norm, and the same vector through both entry points."""
from __future__ import annotations

import numpy as np
import pytest

from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err
from tests.golden.fingerprint import gguf_fingerprint
from tests.test_gpu_decode import logit_tol, report

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["tiny", "tiny-mha", "tiny-q8", "tinyllama"])
def test_embed_matches_reference(name):
    g = load_golden("embed")
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g[f"{name}_fingerprint"].tobytes()
    tol = logit_tol(name)
    with runtime.CudaModel(path, cfg.ctx) as m:
        for key in ("prompt", "one", "long"):
            if f"{name}_{key}_tokens" not in g:
                continue
            toks = g[f"{name}_{key}_tokens"]
            want = g[f"{name}_{key}_embed"]
            got = m.embed(toks)
            err = rel_err(got, want)
            report(name, "embed", tokens=len(toks), max_rel_err=err, tol=tol)
            assert err < tol, key
            assert abs(float(np.linalg.norm(got.astype(np.float64))) - 1.0) < 1e-5
            np.testing.assert_array_equal(m.scheduler_embed(toks), got)


def test_embed_then_decode():
    """The embedding overwrites sequence 0's cache rows 0..n-1, as the
    reference's does; a prompt ingested afterwards decodes the fixture's
    tokens again."""
    name = "tinyllama"
    g = load_golden(name)
    cfg = configs.get(name)
    prompt = [int(t) for t in g["prompt"]]
    with runtime.CudaModel(synth.ensure_gguf(cfg), int(g["ctx"])) as m:
        e1 = m.embed(load_golden("embed")[f"{name}_long_tokens"])
        first = m.prefill(prompt, 0)
        ids = [first] + m.decode_greedy(first, len(prompt), 7)
        assert ids == [int(t) for t in g["ids"][:8]]
        np.testing.assert_array_equal(m.embed(load_golden("embed")[f"{name}_long_tokens"]), e1)


def test_embed_errors():
    cfg = configs.get("tiny")
    path = synth.ensure_gguf(cfg)
    with runtime.CudaModel(path, cfg.ctx) as m:
        with pytest.raises(runtime.SSCudaError):
            m.embed([])
        with pytest.raises(runtime.SSCudaError):
            m.embed([cfg.vocab])
        with pytest.raises(runtime.SSCudaError):
            m.embed([1] * (cfg.ctx + 1))
        m.embed([1, 2, 3])
    with runtime.CudaModel(path, cfg.ctx, flags=runtime.FLAG_MULTI_KERNEL) as m:
        with pytest.raises(runtime.SSCudaError):  # no tiled layout: no many-token step
            m.embed([1, 2, 3])
