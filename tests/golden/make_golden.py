#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the REFERENCE build.

Runs the reference's own CPU path (oracle/_ref, compiled from the PhoneMap
sources by oracle/build_ref.py) on the seeded synthetic GGUF models and records:

* ``<config>.npz`` -- prompt, greedy token IDs (temperature 0) for N steps,
  logits at a few steps, a fingerprint of the GGUF bytes, and the int8 K/V rows
  plus scales of one (layer, position).
* ``sample.npz`` -- the reference's ss_sample draws on the cases of
  ``sample_cases.py``.
* ``quant.npz`` -- the reference's dequantization of every block type it
  handles and its Q4_K matvec, on the inputs of ``quant_cases.py``.
* ``ops.npz`` -- small known-answer vectors of the single ops: Q4_0/Q8_0
  dequantization of seeded blocks (including edge blocks: zero scale, extreme
  nibbles, subnormal/negative scales), dequant-matvec, RMSNorm, RoPE, softmax,
  argmax ties.

Usage: python tests/golden/make_golden.py [fixture ...]   (default: small set)
Needs the reference sources (oracle/build_ref.py finds them) -- fixtures are
committed so the tests never need them.

A fixture is named after its configuration, or after the configuration plus a
suffix when it runs a shorter prompt or starts past position 0 (SPECS below):
the large configurations run a short prompt and a few steps so the reference's
CPU path finishes in minutes, and ``llama3-8b-p600`` starts its prompt at
position 600 -- past the reference's 512-position cap (layer_scheduler.c:202,
430), which the ctx8k build raises -- on a cache whose earlier rows are the
reset zeros on both sides.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from phonemap_b200 import configs, synth  # noqa: E402
from tests.golden.fingerprint import gguf_fingerprint  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# fixture -> (configuration, prompt tokens (None: the configuration's), steps,
# position of the first prompt token)
SPECS = {
    "tiny": ("tiny", None, 24, 0),
    "tiny-mha": ("tiny-mha", None, 20, 0),
    "tiny-q8": ("tiny-q8", None, 20, 0),
    "tinyllama": ("tinyllama", None, 64, 0),
    "llama2-7b": ("llama2-7b", None, 64, 0),
    "llama3-8b": ("llama3-8b", 16, 16, 0),
    "llama3-8b-p600": ("llama3-8b", 8, 8, 600),
    "llama2-13b": ("llama2-13b", 16, 16, 0),
    "llama2-70b-4l": ("llama2-70b-4l", 16, 16, 0),
    "llama2-70b": ("llama2-70b", 8, 8, 0),
}


def make_model_fixture(name: str) -> None:
    cname, nprompt, steps, start = SPECS.get(name, (name, None, 64, 0))
    cfg = configs.get(cname)
    path = synth.ensure_gguf(cfg)
    ref = oracle.RefModel(path, cfg.ctx)
    prompt = synth.prompt_tokens(cfg, nprompt)
    keep = sorted({0, 1, steps // 2, steps - 1})
    ids, all_logits = ref.greedy(prompt, steps, keep_logits=set(range(steps)), start_pos=start)
    kept = {s: all_logits[s] for s in keep}
    # per step: the 4 best token IDs and their logits, and max |logit|
    order = [np.argsort(-all_logits[s], kind="stable")[:4] for s in range(steps)]
    topk_ids = np.array(order, np.int32)
    topk_vals = np.array([all_logits[s][o] for s, o in enumerate(order)], np.float32)
    absmax = np.array([np.abs(all_logits[s]).max() for s in range(steps)], np.float32)
    layer, pos = min(1, cfg.n_layers - 1), start + len(prompt) - 1
    k, v, ks, vs = ref.kv_row(layer, pos)
    np.savez_compressed(
        os.path.join(OUT, f"{name}.npz"),
        prompt=np.array(prompt, np.int32), ids=np.array(ids, np.int32),
        logit_steps=np.array(keep, np.int32),
        logits=np.stack([kept[s] for s in keep]).astype(np.float32),
        fingerprint=np.frombuffer(gguf_fingerprint(path), np.uint8),
        kv_layer=np.int32(layer), kv_pos=np.int32(pos), k_row=k, v_row=v,
        kv_scales=np.array([ks, vs], np.float32), ctx=np.int32(cfg.ctx),
        topk_ids=topk_ids, topk_vals=topk_vals, absmax=absmax,
        config=np.array(cname), start_pos=np.int32(start))
    ref.close()
    print(f"{name}: {steps} steps, ids[:8]={ids[:8]}")


def _blocks_q4(rng, nblk):
    b = np.zeros((nblk, 18), np.uint8)
    d = (rng.standard_normal(nblk) * 0.01).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    b[:, 2:] = rng.integers(0, 256, size=(nblk, 16), dtype=np.uint8)
    # edge blocks: zero scale, all-0x00 / all-0xFF nibbles, negative, subnormal,
    # max-normal fp16 scales
    specials = [0x0000, 0x8000, 0x0001, 0x83FF, 0x7BFF, 0xFBFF, 0x3C00]
    for i, h in enumerate(specials):
        b[i, 0:2] = np.array([h], np.uint16).view(np.uint8)
    b[0, 2:] = 0x00
    b[1, 2:] = 0xFF
    b[2, 2:] = 0x88
    return b


def _blocks_q8(rng, nblk):
    b = np.zeros((nblk, 34), np.uint8)
    d = (rng.standard_normal(nblk) * 0.01).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    b[:, 2:] = rng.integers(0, 256, size=(nblk, 32), dtype=np.uint8)
    specials = [0x0000, 0x8000, 0x0001, 0x83FF, 0x7BFF, 0xFBFF, 0x3C00]
    for i, h in enumerate(specials):
        b[i, 0:2] = np.array([h], np.uint16).view(np.uint8)
    b[0, 2:] = 0x80
    b[1, 2:] = 0x7F
    return b


def make_ops_fixture() -> None:
    import ctypes
    lib = oracle.ref_ops()
    rng = np.random.default_rng(2024)
    fx = {}
    f32p = ctypes.POINTER(ctypes.c_float)
    for name, mk, t in (("q4_0", _blocks_q4, 2), ("q8_0", _blocks_q8, 8)):
        rows, cols = 24, 256
        blocks = mk(rng, rows * cols // 32)
        raw = np.ascontiguousarray(blocks.reshape(-1))
        deq = np.empty(rows * cols, np.float32)
        lib.ssr_dequantize(raw.ctypes.data, deq.ctypes.data_as(f32p), rows * cols, t)
        x = rng.standard_normal(cols).astype(np.float32)
        mv = np.empty(rows, np.float32)
        lib.ssr_dequant_matvec(mv.ctypes.data_as(f32p), raw.ctypes.data,
                               x.ctypes.data_as(f32p), rows, cols, t)
        fx[f"{name}_raw"] = raw
        fx[f"{name}_deq"] = deq
        fx[f"{name}_x"] = x
        fx[f"{name}_mv"] = mv
    halfs = np.array([0x0000, 0x3C00, 0xBC00, 0x3800, 0x0001, 0x03FF, 0x0400, 0x7BFF,
                      0xFBFF, 0x8001, 0x7C00, 0xFC00], np.uint16)
    fx["f16_in"] = halfs
    fx["f16_out"] = np.array([lib.ssr_f16_to_f32(int(h)) for h in halfs], np.float32)
    n = 300
    x = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    out = np.empty(n, np.float32)
    lib.ssr_rmsnorm(out.ctypes.data_as(f32p), x.ctypes.data_as(f32p),
                    w.ctypes.data_as(f32p), n, np.float32(1e-5))
    fx.update(rms_x=x, rms_w=w, rms_out=out)
    nh, nkv, hd = 4, 2, 16
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    fx.update(rope_q_in=q.copy(), rope_k_in=k.copy())
    for pos, theta in ((0, 10000.0), (7, 10000.0), (383, 10000.0), (1000, 500000.0)):
        qq, kk = q.copy(), k.copy()
        lib.ssr_rope(qq.ctypes.data_as(f32p), kk.ctypes.data_as(f32p), nh, nkv, hd, hd, pos,
                     np.float32(theta))
        fx[f"rope_q_{pos}"] = qq
        fx[f"rope_k_{pos}"] = kk
    s = (rng.standard_normal(77) * 3).astype(np.float32)
    fx["softmax_in"] = s.copy()
    lib.ssr_softmax(s.ctypes.data_as(f32p), len(s))
    fx["softmax_out"] = s
    ties = np.array([1.0, 5.0, 2.0, 5.0, 5.0, -1.0], np.float32)
    fx["argmax_ties_in"] = ties
    fx["argmax_ties_out"] = np.int32(lib.ssr_argmax(ties.ctypes.data_as(f32p), len(ties)))
    np.savez_compressed(os.path.join(OUT, "ops.npz"), **fx)
    print("ops: written")


def make_argmax_fixture() -> None:
    """argmax.npz: expected ss_argmax results of the edge-case arrays (the big
    ones are regenerated by the tests from the same seed) and the reference's
    greedy token for each crafted ``tiny`` model (tests/golden/crafted.py)."""
    import ctypes
    import tempfile

    from tests.golden import crafted
    lib = oracle.ref_ops()
    f32p = ctypes.POINTER(ctypes.c_float)
    fx = {}
    for k, a in crafted.argmax_arrays().items():
        fx[f"want_{k}"] = np.int32(lib.ssr_argmax(a.ctypes.data_as(f32p), a.size))
        if a.size < 64:
            fx[f"in_{k}"] = a
    cfg = configs.get("tiny")
    src = synth.ensure_gguf(cfg)
    prompt = synth.prompt_tokens(cfg)
    with tempfile.TemporaryDirectory() as td:
        for case in crafted.CASES:
            dst = os.path.join(td, f"tiny-{case}.gguf")
            crafted.make_crafted(case, src, dst)
            ref = oracle.RefModel(dst, cfg.ctx)
            lg = ref.prefill(prompt, 0)
            fx[f"model_{case}"] = np.int32(lib.ssr_argmax(lg.ctypes.data_as(f32p), lg.size))
            fx[f"model_{case}_nnan"] = np.int32(np.isnan(lg).sum())
            fx[f"model_{case}_nzero"] = np.int32((lg == 0).sum())
            ref.close()
            print(case, int(fx[f"model_{case}"]), "nan", int(fx[f"model_{case}_nnan"]),
                  "zeros", int(fx[f"model_{case}_nzero"]), "max", np.nanmax(lg))
    np.savez_compressed(os.path.join(OUT, "argmax.npz"), **fx)
    print("argmax: written", {k: int(v) for k, v in fx.items() if k.startswith("want_")})


EMBED_CONFIGS = ("tiny", "tiny-mha", "tiny-q8", "tinyllama")


def embed_prompts(cfg) -> dict:
    """The token lists embed.npz holds for a configuration: its prompt, one
    token, and (where the context allows) 70 tokens -- more than one pass of
    the GPU's 32-token step."""
    p = [int(t) for t in synth.prompt_tokens(cfg)]
    out = {"prompt": p, "one": p[:1]}
    if cfg.ctx >= 80:
        rng = np.random.default_rng(99)
        out["long"] = [int(t) for t in rng.integers(0, cfg.vocab, size=70)]
    return out


def make_embed_fixture() -> None:
    """embed.npz: ss_scheduler_embed's vector (layer_scheduler.c:805-915),
    from the reference build, for each configuration's token lists."""
    fx = {}
    for cname in EMBED_CONFIGS:
        cfg = configs.get(cname)
        path = synth.ensure_gguf(cfg)
        fx[f"{cname}_fingerprint"] = np.frombuffer(gguf_fingerprint(path), np.uint8)
        for key, toks in embed_prompts(cfg).items():
            ref = oracle.RefModel(path, cfg.ctx)
            fx[f"{cname}_{key}_tokens"] = np.array(toks, np.int32)
            fx[f"{cname}_{key}_embed"] = ref.embed(toks).astype(np.float32)
            ref.close()
    np.savez_compressed(os.path.join(OUT, "embed.npz"), **fx)
    print(f"embed: {sorted(k for k in fx if k.endswith('_embed'))}")


def make_sample_fixture() -> None:
    """sample.npz: the reference's ss_sample (tensor.c:363-451) on every case of
    tests/golden/sample_cases.py -- DRAWS chained draws each: the tokens, the
    RNG states after each draw, and a digest of the logits drawn from."""
    from tests.golden import sample_cases as sc
    fx = {}
    for name, (make, *_rest) in sc.CASES.items():
        toks, states = sc.draws(oracle.ref_sample, name)
        fx[f"{name}/digest"] = np.frombuffer(sc.digest(make()), np.uint8)
        fx[f"{name}/tokens"] = np.array(toks, np.int32)
        fx[f"{name}/states"] = np.array(states, np.uint64)
    np.savez_compressed(os.path.join(OUT, "sample.npz"), **fx)
    print(f"sample: {len(sc.CASES)} cases")


def make_quant_fixture() -> None:
    """quant.npz: the reference's ss_dequantize (quantize.c:389-442) on the
    seeded blocks of tests/golden/quant_cases.py, every type it handles, and
    its ss_dequant_matvec (quantize.c:446-494) on the Q4_K matrix there."""
    import ctypes

    from tests.golden import quant_cases as qc
    lib = oracle.ref_ops()
    f32p = ctypes.POINTER(ctypes.c_float)
    fx = {}
    for t in qc.TYPES:
        raw, n = qc.blocks(t)
        out = np.empty(n, np.float32)
        lib.ssr_dequantize(raw.ctypes.data, out.ctypes.data_as(f32p), n, t)
        fx[f"{qc.NAMES[t]}/blocks"] = raw
        fx[f"{qc.NAMES[t]}/values"] = out
    raw, x = qc.q4k_matrix()
    rows, cols = 48, 1024
    out = np.empty(rows, np.float32)
    lib.ssr_dequant_matvec(out.ctypes.data_as(f32p), raw.ctypes.data, x.ctypes.data_as(f32p), rows, cols, 12)
    fx["q4k_mv/w"], fx["q4k_mv/x"], fx["q4k_mv/out"] = raw, x, out
    np.savez_compressed(os.path.join(OUT, "quant.npz"), **fx)
    print(f"quant: {sorted(qc.NAMES.values())}")


def main() -> int:
    if not oracle.ref_available() and not oracle.build_ref():
        print("reference build unavailable", file=sys.stderr)
        return 2
    names = sys.argv[1:] or ["ops", "tiny", "tiny-mha", "tiny-q8", "tinyllama"]
    for n in names:
        if n == "ops":
            make_ops_fixture()
        elif n == "argmax":
            make_argmax_fixture()
        elif n == "embed":
            make_embed_fixture()
        elif n == "sample":
            make_sample_fixture()
        elif n == "quant":
            make_quant_fixture()
        else:
            make_model_fixture(n)
    return 0


if __name__ == "__main__":
    sys.exit(main())
