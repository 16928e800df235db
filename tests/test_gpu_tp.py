"""Tensor-parallel decode (2/4/8 GPUs, one process per GPU, NCCL) against the
reference's golden fixtures, with the single-GPU tolerances: greedy token IDs
identical (a divergence only where the reference's own top-2 lie within the
logit tolerance), logits within the tolerance, and rank 0's int8 K/V row --
its kv heads, quantised with the scale of the whole kv_dim after the max
all-reduce -- within one quantisation step of the reference's.  Sharding
changes only the fp32 summation order of the O and down projections.  Both
step implementations: the persistent kernel (exchanges through peer memory
inside the kernel) and the multi-kernel graph (NCCL between kernels)."""
from __future__ import annotations

import numpy as np
import pytest

from phonemap_b200 import configs, runtime, synth, tp
from tests.conftest import load_golden, rel_err
from tests.test_gpu_decode import PATHS, _acceptable_choice, logit_tol

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _divisible(cfg, n: int) -> bool:
    return (cfg.n_heads % n == 0 and cfg.n_kv_heads % n == 0 and cfg.ffn % (32 * n) == 0
            and cfg.vocab % n == 0)


CASES = [(2, "tiny"), (2, "tiny-mha"), (2, "tiny-q8"), (2, "tinyllama"), (2, "llama2-7b"),
         (4, "tinyllama"), (4, "llama2-7b"), (8, "llama2-7b"), (2, "llama3-8b"), (4, "llama3-8b"),
         (8, "llama3-8b")]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("n,name", CASES, ids=[f"tp{n}-{m}" for n, m in CASES])
def test_tp_greedy_parity(n, name, path):
    if _gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    cfg = configs.get(name)
    assert _divisible(cfg, n)
    g = load_golden(name)
    tol = logit_tol(name)
    prompt = [int(t) for t in g["prompt"]]
    ref = [int(t) for t in g["ids"]]
    r = tp.greedy(synth.ensure_gguf(cfg), int(g["ctx"]), prompt, len(ref), n, flags=PATHS[path],
                  kv_at=(int(g["kv_layer"]), int(g["kv_pos"])))
    assert r["stats"]["persistent"] == (0 if PATHS[path] & runtime.FLAG_MULTI_KERNEL else 1)
    ids, logits = r["ids"], r["logits"]
    first = next((i for i, (a, b) in enumerate(zip(ids, ref)) if a != b), len(ref))
    for i, s in enumerate(g["logit_steps"]):
        if int(s) <= first:
            assert rel_err(logits[int(s)], g["logits"][i]) < tol, f"step {s}"
    if first < len(ref):
        assert _acceptable_choice(g, first, ids[first], tol), f"diverged at step {first}"
    # the device-resident loop gives the host loop's tokens
    assert r["loop_ids"] == ids
    k, v, ks, vs = r["kv_row0"]
    kvd_l = cfg.kv_dim // n
    assert np.abs(k.astype(int) - g["k_row"][:kvd_l]).max() <= 1
    assert np.abs(v.astype(int) - g["v_row"][:kvd_l]).max() <= 1
    np.testing.assert_allclose([ks, vs], g["kv_scales"], rtol=max(1e-3, tol))


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", ["tiny", "tinyllama"])
def test_tp_teacher_forced(name, path):
    """Every step fed the reference's token: logits at the reference's top-4
    within the tolerance, argmax the reference's wherever its margin exceeds
    the tolerance."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = configs.get(name)
    g = load_golden(name)
    tol = logit_tol(name)
    ref = [int(t) for t in g["ids"]]
    r = tp.greedy(synth.ensure_gguf(cfg), int(g["ctx"]), [int(t) for t in g["prompt"]], len(ref), 2,
                  teacher=ref, flags=PATHS[path])
    for s in range(len(ref)):
        top, vals, am = g["topk_ids"][s], g["topk_vals"][s], float(g["absmax"][s])
        assert np.abs(r["logits"][s][top] - vals).max() / am < tol, f"step {s}"
        if float(vals[0] - vals[1]) > tol * am:
            assert r["ids"][s] == ref[s], f"step {s}"


@pytest.mark.parametrize("path", PATHS)
def test_tp_sampling(path):
    """Sampling under tensor parallelism: every rank gathers the logits and
    draws the same token.  ss_cuda_decode_sample equals a host loop of
    ss_cuda_sample + ss_cuda_forward; each of those draws is the restatement's
    (the GPU's exponential) on the step's gathered logits and RNG state; every
    rank drew the same tokens."""
    import oracle
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = configs.get("tinyllama")
    g = load_golden("tinyllama")
    prompt = [int(t) for t in g["prompt"]]
    t, p, k, seed = 0.7, 0.9, 40, 0x9E3779B97F4A7C15
    r = tp.greedy(synth.ensure_gguf(cfg), int(g["ctx"]), prompt, 16, 2, flags=PATHS[path],
                  sample=(t, p, k, seed))
    sd = r["sampled"]
    assert sd["dev_ids"] == sd["ids"]
    assert sd["dev_state"] == sd["states"][-1]
    for i, tok in enumerate(sd["ids"]):
        assert oracle.sample(sd["logits"][i], t, p, k, sd["states"][i], 1) == (tok, sd["states"][i + 1])
    for dev_ids, host_ids in r["sampled_ids_other"]:
        assert dev_ids == sd["dev_ids"] and host_ids == sd["ids"]
