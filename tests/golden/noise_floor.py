#!/usr/bin/env python3
"""Measure a configuration's parity noise floor -- TEST INFRASTRUCTURE.

Runs the oracle restatement twice on the same seeded model and prompt: once in
the reference's own arithmetic order (bit-identical to the reference, see
test_oracle_golden.py) and once with every quantized matvec summed in a
GPU-shaped blocked order (oracle sso_set_dot_order(1)) -- two equally valid
fp32 evaluations of the same math.  How far their logits differ is the floor
below which no implementation that sums in a different order can be expected
to agree with the reference; the int8 KV cache (roundf per value,
layer_scheduler.c:116) amplifies last-bit differences, so this floor grows with
depth and prompt length.

Records {config: {"prefill_inf_rel", "prefill_l2_rel", "steps", "max_step_inf_rel"}}
in tests/golden/noise_floor.json.  The decode steps are teacher-forced with the
reference's golden tokens.

Usage: python tests/golden/noise_floor.py [config ...] [--steps N]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from phonemap_b200 import configs, synth  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "noise_floor.json")


def measure(name: str, steps: int) -> dict:
    g = np.load(os.path.join(os.path.dirname(OUT), f"{name}.npz"))
    cfg = configs.get(str(g["config"]) if "config" in g.files else name)
    start = int(g["start_pos"]) if "start_pos" in g.files else 0
    m = oracle.OracleModel(synth.ensure_gguf(cfg), int(g["ctx"]))
    m.set_dot_order(1)
    prompt = [int(t) for t in g["prompt"]]
    ref_ids = [int(t) for t in g["ids"]]
    logits = m.prefill(prompt, start)
    ref0 = g["logits"][0]
    d = logits.astype(np.float64) - ref0
    res = {"prefill_inf_rel": float(np.abs(d).max() / np.abs(ref0).max()),
           "prefill_l2_rel": float(np.linalg.norm(d) / np.linalg.norm(ref0))}
    worst = res["prefill_inf_rel"]
    steps = min(steps, len(ref_ids))
    kept = {int(s): i for i, s in enumerate(g["logit_steps"])}
    for s in range(1, steps):
        logits = m.forward(ref_ids[s - 1], start + len(prompt) + s - 1)
        if s in kept:
            ref = g["logits"][kept[s]]
            worst = max(worst, float(np.abs(logits - ref).max() / np.abs(ref).max()))
    res["steps"] = steps
    res["max_step_inf_rel"] = worst
    m.close()
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("configs", nargs="*", default=["tiny", "tinyllama"])
    ap.add_argument("--steps", type=int, default=64)
    args = ap.parse_args()
    data = json.load(open(OUT)) if os.path.exists(OUT) else {}
    for name in args.configs:
        data[name] = measure(name, args.steps)
        print(name, data[name], flush=True)
        with open(OUT, "w") as f:
            json.dump(data, f, indent=1, sort_keys=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
