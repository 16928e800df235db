"""GPU decode parity against the reference (golden fixtures made by the
reference's own CPU path): greedy token IDs identical, logits within 1e-2 of
max |logit| (or twice the configuration's measured noise floor where that is
larger, see logit_tol), int8 KV rows within one quantisation step.  Both step
implementations are checked: the persistent single kernel (the default) and
the multi-kernel CUDA graph (SS_CUDA_FLAG_MULTI_KERNEL)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from phonemap_b200 import configs, runtime, synth
from tests.conftest import load_golden, rel_err
from tests.golden.fingerprint import gguf_fingerprint

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-2
PATHS = {"persistent": 0, "multi-kernel": runtime.FLAG_MULTI_KERNEL}


def fixture_config(g: dict, name: str):
    """The configuration a fixture was made from (its own name for the older
    fixtures) and the position of its first prompt token."""
    cname = str(g["config"]) if "config" in g else name
    return configs.get(cname), int(g["start_pos"]) if "start_pos" in g else 0


def report(name: str, path: str, **kw) -> None:
    """Parity figures of one run: printed, and appended as a JSON line to
    $SS_PARITY_REPORT when that is set."""
    import json
    import os
    rec = {"fixture": name, "path": path, **kw}
    print("parity", json.dumps(rec))
    out = os.environ.get("SS_PARITY_REPORT")
    if out:
        with open(out, "a") as f:
            f.write(json.dumps(rec) + "\n")


def _run(name: str, flags: int = 0):
    g = load_golden(name)
    cfg, start = fixture_config(g, name)
    path = synth.ensure_gguf(cfg)
    assert gguf_fingerprint(path) == g["fingerprint"].tobytes()
    m = runtime.CudaModel(path, int(g["ctx"]), flags=flags)
    if flags & runtime.FLAG_MULTI_KERNEL:
        assert m.stats()["persistent"] == 0
    elif not m.stats()["persistent"]:
        # a shape beyond the persistent kernel's limits (the 70B FFN width,
        # 896 column blocks, on one GPU) runs the multi-kernel step, which the
        # multi-kernel parameter of the same test covers
        m.close()
        pytest.skip(f"{name}: persistent step not eligible on one GPU")
    prompt = [int(t) for t in g["prompt"]]
    steps = len(g["ids"])
    logits = {}
    buf = np.empty(m.vocab, np.float32)
    ids = [m.prefill(prompt, start, logits=buf)]
    logits[0] = buf.copy()
    pos = start + len(prompt)
    for s in range(1, steps):
        ids.append(m.forward(ids[-1], pos, logits=buf))
        logits[s] = buf.copy()
        pos += 1
    return g, m, ids, logits


# Tolerance per configuration.  The north-star bar is 1e-2 of max |logit|.  The
# int8 KV cache rounds every K/V value with roundf (layer_scheduler.c:116), so a
# last-bit difference anywhere upstream can flip a value by one step, and the
# reference's own CPU arithmetic summed in another (equally valid) fp32 order
# already moves its logits; tests/golden/noise_floor.json records that floor
# per configuration (oracle, sso_set_dot_order(1)).  Where twice the floor
# exceeds 1e-2 (the 32-layer Llama-2-7B shape with a 128-token prompt), the
# tolerance is twice the floor, and the report says so.
FIXTURES = ["tiny", "tiny-mha", "tiny-q8", "tinyllama", "llama2-7b", "llama3-8b",
            "llama3-8b-p600", "llama2-13b", "llama2-70b-4l"]


def logit_tol(name: str) -> float:
    import json
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "noise_floor.json")
    floor = json.load(open(path)).get(name, {}).get("max_step_inf_rel", 0.0)
    return max(LOGIT_RTOL, 2.0 * floor)


def _acceptable_choice(g, step: int, token: int, tol: float) -> bool:
    """`token` is a valid greedy choice at `step` if its reference logit is within
    the logit tolerance of the reference maximum (it must be one of the
    reference's recorded top 4)."""
    top = [int(t) for t in g["topk_ids"][step]]
    if token not in top:
        return False
    vals = g["topk_vals"][step]
    return float(vals[0] - vals[top.index(token)]) <= tol * float(g["absmax"][step])


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", FIXTURES)
def test_greedy_parity(name, path):
    """Free-running greedy decode: identical to the reference's token IDs; a
    divergence is only accepted at a step where the reference's own top-2 lie
    within the logit tolerance, and the GPU's choice must be acceptable there.
    Logits agree within the tolerance at every recorded step before it."""
    tol = logit_tol(name)
    g, m, ids, logits = _run(name, PATHS[path])
    ref = [int(t) for t in g["ids"]]
    first = next((i for i, (a, b) in enumerate(zip(ids, ref)) if a != b), len(ref))
    errs = {int(s): rel_err(logits[int(s)], g["logits"][i])
            for i, s in enumerate(g["logit_steps"]) if int(s) <= first}
    report(name, path, mode="free-running", steps=len(ref), first_divergence=first,
           identical_ids=first == len(ref), max_rel_logit_err=max(errs.values()),
           rel_logit_err_by_step=errs, tol=tol, meets_north_star_1e2=max(errs.values()) < 1e-2)
    for s, e in errs.items():
        assert e < tol, f"step {s}"
    if first < len(ref):
        assert _acceptable_choice(g, first, ids[first], tol), f"diverged at step {first}"
    m.close()


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", FIXTURES)
def test_teacher_forced_parity(name, path):
    """Every step fed the reference's own token: the GPU logits at the
    reference's top-4 tokens agree within the tolerance, and the GPU's argmax
    is the reference's at every step whose reference margin exceeds the
    tolerance (elsewhere it must be an acceptable choice)."""
    tol = logit_tol(name)
    g = load_golden(name)
    cfg, start = fixture_config(g, name)
    gpath = synth.ensure_gguf(cfg)
    ref = [int(t) for t in g["ids"]]
    worst = 0.0
    with runtime.CudaModel(gpath, int(g["ctx"]), flags=PATHS[path]) as m:
        buf = np.empty(m.vocab, np.float32)
        prompt = [int(t) for t in g["prompt"]]
        got = m.prefill(prompt, start, logits=buf)
        # int8 K/V row written by the prompt: within one quantisation step
        k, v, ks, vs = m.kv_row(int(g["kv_layer"]), int(g["kv_pos"]))
        assert np.abs(k.astype(int) - g["k_row"]).max() <= 1
        assert np.abs(v.astype(int) - g["v_row"]).max() <= 1
        # the share of exactly equal int8 values: a last-bit difference upstream
        # moves a value across a roundf .5 boundary, more often the deeper the
        # configuration's noise floor (4-layer 70B shape: about 2% differ by one)
        same = 0.98 if logit_tol(name) <= LOGIT_RTOL else 0.95
        assert (k == g["k_row"]).mean() > same and (v == g["v_row"]).mean() > same
        np.testing.assert_allclose([ks, vs], g["kv_scales"], rtol=max(1e-3, tol))
        for s in range(len(ref)):
            if s > 0:
                got = m.forward(ref[s - 1], start + len(prompt) + s - 1, logits=buf)
            top, vals, am = g["topk_ids"][s], g["topk_vals"][s], float(g["absmax"][s])
            worst = max(worst, float(np.abs(buf[top] - vals).max() / am))
            assert np.abs(buf[top] - vals).max() / am < tol, f"step {s}"
            if float(vals[0] - vals[1]) > tol * am:
                assert got == ref[s], f"step {s}"
            else:
                assert _acceptable_choice(g, s, got, tol), f"step {s}"
    report(name, path, mode="teacher-forced", steps=len(ref), max_rel_top4_err=worst, tol=tol)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", ["tiny", "tinyllama"])
def test_device_loop_equals_host_loop(name, path):
    """ss_cuda_decode_greedy (tokens fed back on the device, no host round trip
    between steps) produces the same tokens as step-by-step ss_cuda_forward."""
    g, m, ids, _ = _run(name, PATHS[path])
    m.reset()
    prompt = [int(t) for t in g["prompt"]]
    first = m.prefill(prompt, 0)
    dev = [first] + m.decode_greedy(first, len(prompt), len(ids) - 1)
    assert dev == ids
    m.close()


def test_no_pdl_no_graph_same_result():
    """PDL/graph chaining of the multi-kernel step changes scheduling only,
    never results."""
    multi = runtime.FLAG_MULTI_KERNEL
    _, m1, ids1, lg1 = _run("tiny", flags=multi)
    _, m2, ids2, lg2 = _run("tiny", flags=multi | runtime.FLAG_NO_PDL | runtime.FLAG_NO_GRAPH)
    assert ids1 == ids2
    for s in lg1:
        np.testing.assert_array_equal(lg1[s], lg2[s])
    m1.close()
    m2.close()


@pytest.mark.parametrize("name", ["tiny", "tinyllama"])
def test_persistent_matches_multi_kernel(name):
    """The two step implementations agree with each other to fp32 rounding
    (different summation orders) at every recorded step, on the same tokens."""
    g = load_golden(name)
    cfg = configs.get(name)
    gpath = synth.ensure_gguf(cfg)
    prompt = [int(t) for t in g["prompt"]]
    ref = [int(t) for t in g["ids"]]
    with runtime.CudaModel(gpath, int(g["ctx"])) as a, \
            runtime.CudaModel(gpath, int(g["ctx"]), flags=runtime.FLAG_MULTI_KERNEL) as b:
        la = np.empty(a.vocab, np.float32)
        lb = np.empty(b.vocab, np.float32)
        a.prefill(prompt, 0, logits=la)
        b.prefill(prompt, 0, logits=lb)
        assert rel_err(la, lb) < logit_tol(name)
        for s in range(1, min(len(ref), 16)):
            a.forward(ref[s - 1], len(prompt) + s - 1, logits=la)
            b.forward(ref[s - 1], len(prompt) + s - 1, logits=lb)
            assert rel_err(la, lb) < logit_tol(name), f"step {s}"


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


@pytest.mark.parametrize("name", ["tiny-q8", "tinyllama"])
def test_deterministic_across_runs(name):
    """Bitwise-identical logits across runs (no order-dependent atomics)."""
    _, m1, ids1, lg1 = _run(name)
    _, m2, ids2, lg2 = _run(name)
    assert ids1 == ids2
    for s in lg1:
        np.testing.assert_array_equal(lg1[s], lg2[s])


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("case", ["nan0", "zeros", "allzero", "negzero"])
def test_argmax_rule_through_lm_head(case, path, tmp_path):
    """The greedy token of the lm_head epilogue follows ss_argmax
    (tensor.c:318-328) on crafted lm_head rows (tests/golden/crafted.py): a
    NaN logit at index 0, ties between equal rows, +0.0 against -0.0.  The
    expected token is the reference's own on the same bytes."""
    from tests.golden import crafted
    want = int(load_golden("argmax")[f"model_{case}"])
    cfg = configs.get("tiny")
    dst = str(tmp_path / f"tiny-{case}.gguf")
    crafted.make_crafted(case, synth.ensure_gguf(cfg), dst)
    with runtime.CudaModel(dst, cfg.ctx, flags=PATHS[path]) as m:
        assert m.prefill(synth.prompt_tokens(cfg), 0) == want


@pytest.mark.parametrize("phase_of", ["qkv0", "down1", "head"])
def test_bounded_wait_expires_then_reset_recovers(phase_of):
    """A device wait that runs out (the producer withholds one weight stage:
    ss_cuda_test_fail_next_step) ends the step with SS_CUDA_ERROR_BACKEND and
    the ring-wait error bit -- no fault, no hang -- and after ss_cuda_reset
    the same context decodes the reference's tokens again."""
    g = load_golden("tiny")
    cfg = configs.get("tiny")
    L = cfg.n_layers
    phase = {"qkv0": 1, "down1": 5 * 1 + 1 + 4, "head": 5 * L + 1}[phase_of]
    prompt = [int(t) for t in g["prompt"]]
    ref = [int(t) for t in g["ids"]]
    with runtime.CudaModel(synth.ensure_gguf(cfg), int(g["ctx"])) as m:
        first = m.prefill(prompt, 0)
        assert first == ref[0]
        m.test_fail_next_step(phase)
        with pytest.raises(runtime.SSCudaError) as e:
            m.forward(first, len(prompt))
        assert e.value.code == -7 and "ring wait" in str(e.value)
        m.reset()
        first = m.prefill(prompt, 0)
        ids = [first] + m.decode_greedy(first, len(prompt), 7)
        assert ids == ref[:8]


@pytest.mark.parametrize("name", ["tiny", "tiny-mha", "tiny-q8", "tinyllama"])
def test_batched_prefill_matches_replay(name):
    """The prompt through the many-token tensor-core step (32 tokens per pass)
    against the decode step replayed per token (SS_CUDA_FLAG_STEP_PREFILL, the
    reference's order): last-token logits within the configuration's
    tolerance, the int8 K/V rows of every prompt position within one step,
    and the same greedy continuation."""
    g = load_golden(name)
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    prompt = [int(t) for t in g["prompt"]]
    # a prompt longer than one pass where the context allows it
    long_prompt = (prompt * 40)[:min(70, cfg.ctx - 10)]
    tol = logit_tol(name)
    with runtime.CudaModel(path, cfg.ctx) as a, \
            runtime.CudaModel(path, cfg.ctx, flags=runtime.FLAG_STEP_PREFILL) as b:
        for pr in (prompt, long_prompt):
            a.reset()
            b.reset()
            la = np.empty(a.vocab, np.float32)
            lb = np.empty(b.vocab, np.float32)
            ta = a.prefill(pr, 0, logits=la)
            tb = b.prefill(pr, 0, logits=lb)
            assert rel_err(la, lb) < tol
            for pos in (0, len(pr) // 2, len(pr) - 1):
                for layer in (0, cfg.n_layers - 1):
                    ka, va, ksa, vsa = a.kv_row(layer, pos)
                    kb, vb, ksb, vsb = b.kv_row(layer, pos)
                    assert np.abs(ka.astype(int) - kb).max() <= 1
                    assert np.abs(va.astype(int) - vb).max() <= 1
                    np.testing.assert_allclose([ksa, vsa], [ksb, vsb], rtol=1e-3)
            if ta == tb:
                assert a.decode_greedy(ta, len(pr), 6) == b.decode_greedy(tb, len(pr), 6)
