"""GPU: the allocation-free greedy argmax, ss_cuda_argmax_noalloc.

It exists for callers that cannot allocate device memory at the point where
they need a greedy token (for example while a stream is being captured into a
CUDA graph, where cudaMalloc is not allowed).  Its scratch is a fixed array in
the library's device image instead of context-allocated memory, so this file
checks it against the existing path: the argmax ss_cuda_forward returns for the
same logits (computed by the lm_head kernel with its context's scratch), on two
calls in a row, since every call reuses the array the previous call left
behind.  Device buffers come from torch (plumbing only).  Collected last so a
failure here does not hide the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest

from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden
from tests.golden import crafted

pytestmark = pytest.mark.gpu


def _noalloc(values: np.ndarray) -> int:
    import torch
    d_v = torch.from_numpy(np.ascontiguousarray(values, np.float32)).cuda()
    d_i = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    runtime.argmax_noalloc(d_v.data_ptr(), d_v.numel(), d_i.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    return int(d_i.item())


def test_matches_existing_argmax_twice():
    """Two consecutive steps: the no-alloc argmax of the step's logits equals
    the argmax ss_cuda_forward returned for them."""
    cfg = configs.get("tiny")
    prompt = synth.prompt_tokens(cfg)
    with runtime.CudaModel(synth.ensure_gguf(cfg), cfg.ctx, device=0) as m:
        logits = np.empty(m.vocab, np.float32)
        tok = m.prefill(prompt, 0, logits=logits)
        first = _noalloc(logits)
        assert first == tok
        tok2 = m.forward(tok, len(prompt), logits=logits)
        second = _noalloc(logits)
        assert second == tok2


def test_ties_large_and_sizes():
    """Lowest index wins ties; a multi-CTA input (more than one partial per
    call); the size limit is reported, not run."""
    ties = np.zeros(5000, np.float32)
    ties[[17, 4000, 4999]] = 3.0
    assert _noalloc(ties) == 17
    rng = np.random.default_rng(5)
    big = rng.standard_normal(1 << 20).astype(np.float32)
    assert _noalloc(big) == int(np.argmax(big))
    big[[1000, 700000]] = big.max() + 1.0
    assert _noalloc(big) == 1000
    # refused before anything is enqueued: too large, empty, NULL pointers
    with pytest.raises(runtime.SSCudaError):
        runtime.argmax_noalloc(1, (1 << 22) + 1, 1)
    with pytest.raises(runtime.SSCudaError):
        runtime.argmax_noalloc(1, 0, 1)
    with pytest.raises(runtime.SSCudaError):
        runtime.argmax_noalloc(0, 16, 1)
    with pytest.raises(runtime.SSCudaError):
        runtime.argmax_noalloc(1, 16, 0)


def test_reference_rule_edge_cases():
    """The reference's scan rule (first maximum; -0.0 ties +0.0; NaN after
    index 0 never wins; NaN at index 0 keeps index 0) on the cases whose
    expected index the reference's own ss_argmax gave (tests/golden/argmax.npz),
    including 4,194,304 values -- the size limit, every partial slot in use."""
    g = load_golden("argmax")
    for name, values in crafted.argmax_arrays().items():
        assert _noalloc(values) == int(g[f"want_{name}"]), name
