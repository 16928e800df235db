"""The reference's own scheduler with this repository's CUDA backend plugged
into its dispatch, as a maintainer would (oracle/build_ref.py builds
oracle/_ref/libss_ref_cuda.so from the reference sources with the
INTEGRATION.md section 4 hook: a cuda_ctx next to metal_ctx and an
SS_HAS_CUDA branch in ss_matmul_dispatch, layer_scheduler.c:248-279).  The
reference's prefill/forward then run every Q4_0/Q8_0/F32 projection through
ss_cuda_matvec_q4_0 / _q8_0 / ss_cuda_matvec; the greedy tokens and logits
must match the reference's own CPU run (the golden fixtures) within the
configuration's tolerance, and the backend must have served the matvecs."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err
from tests.test_gpu_decode import _acceptable_choice, logit_tol, report

pytestmark = pytest.mark.gpu

HOOKED = os.path.join(oracle.REF_DIR, "libss_ref_cuda.so")


@pytest.mark.skipif(not os.path.exists(HOOKED), reason="integration build absent (oracle/build_ref.py)")
@pytest.mark.parametrize("name", ["tiny", "tiny-q8", "tinyllama"])
def test_reference_scheduler_on_cuda_backend(name):
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    tol = logit_tol(name)
    ref_ids = [int(t) for t in g["ids"]]
    steps = min(len(ref_ids), 24)
    with runtime.CudaModel(None) as backend:  # an op-level context, as ss_metal_init makes
        ref = oracle.RefModel(path, int(g["ctx"]), cuda_hook=True)
        ref.attach_cuda(backend._h)
        ids, kept = ref.greedy([int(t) for t in g["prompt"]], steps,
                               keep_logits=set(int(s) for s in g["logit_steps"]))
        ref.attach_cuda(None)
        ref.close()
        served = backend.stats()["matvecs_run"]
    # every projection of every layer and the lm_head, for the prompt and each step
    per_token = 7 * cfg.n_layers + 1
    assert served >= per_token * steps, served
    first = next((i for i, (a, b) in enumerate(zip(ids, ref_ids)) if a != b), steps)
    errs = {s: rel_err(kept[s], g["logits"][i]) for i, s in enumerate(int(v) for v in g["logit_steps"])
            if s in kept and s <= first}
    report(name, "reference scheduler + CUDA matvecs", mode="free-running", steps=steps,
           first_divergence=first, max_rel_logit_err=max(errs.values()), tol=tol, matvecs=served)
    for s, e in errs.items():
        assert e < tol, f"step {s}"
    if first < steps:
        assert _acceptable_choice(g, first, ids[first], tol), f"diverged at step {first}"
