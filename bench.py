#!/usr/bin/env python3
"""Decode throughput of SlipStream's per-token loop on B200.

One *step* = one greedy decode token of the workload (batch 1): embedding, all
layers (RMSNorm, Q/K/V GEMV + RoPE, int8-KV attention, O GEMV, RMSNorm,
gate/up GEMV + SwiGLU, down GEMV), final RMSNorm, lm_head, argmax -- one CUDA
graph replay.  Default workload: the Llama-2-7B-shaped Q4_0 model, prompt of
128 seeded tokens, greedy decode at batch 1, ctx 2048 (the configuration the
headline metric is quoted on).  The weights (3.7 GB per step) are far larger
than L2, so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  --impl reference times the reference's own CPU
path (oracle/_ref, or the repository's C restatement when the reference build is
absent) on the host cores instead.  With --gpus N (torchrun, one rank per GPU)
the N ranks decode the same sequence tensor-parallel (heads, FFN rows and
vocabulary split N ways, NCCL all-reduces between the kernels): strong
scaling, value = the sequence's tokens/s; --replicas instead decodes an
independent replica per GPU (weak scaling).  Time is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))

NVML_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="llama2-7b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sample", default="0.7,0.9,40",
                    help="temperature,top_p,top_k of the sampled-decode measurement reported beside "
                         "the greedy one (one GPU; default: the reference's ss_default_params, "
                         "engine.c:42-51); 'off' skips it")
    ap.add_argument("--profile-kernel", default=None,
                    choices=["qkv", "attention", "o", "gate_up", "down", "lm_head", "step",
                             "product_gate_up", "product_qkv_l2"],
                    help="time one step kernel in isolation instead of the decode loop "
                         "(qkv..lm_head need --multi-kernel; step = one whole decode step)")
    ap.add_argument("--multi-kernel", action="store_true",
                    help="run the step as 2 + 5*layers kernels (CUDA graph) instead of the "
                         "persistent single kernel")
    ap.add_argument("--hbm-budget-layers", type=float, default=None,
                    help="HBM budget for the layers' weights, in layers (layer streaming); "
                         "default 4 for llama2-13b (its configuration), else all resident")
    ap.add_argument("--replicas", action="store_true",
                    help="with --gpus N: N independent replicas instead of one tensor-parallel group")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences decoded together per GPU (the many-token tensor-core step; "
                         "with --gpus N, N independent replicas of B sequences)")
    return ap.parse_args()


# --------------------------------------------------------------------- helpers

def hbm_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def read_profile_traffic(kernel: str, config: str):
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every ~10 ms."""

    def __init__(self, device_index: int):
        self.samples = []  # (t, sm_mhz, reasons_bits)
        self.window = None
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = self._handle(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

    def _handle(self, idx):
        import torch
        nv = self._nv
        try:
            uuid = str(torch.cuda.get_device_properties(idx).uuid)
            return nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                idx = int(vis.split(",")[idx])
            return nv.nvmlDeviceGetHandleByIndex(idx)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, r))
            except Exception:
                pass
            time.sleep(0.01)

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join(timeout=1)

    def summary(self):
        if self._h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        t0, t1 = self.window or (0, float("inf"))
        inside = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-5:]
        bits = 0
        for s in inside:
            bits |= s[2]
        reasons = [n for b, n in NVML_REASONS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[1] for s in inside) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside)}


def cpu_reference_run(cfg, path, n_max, budget_s=20.0, start_pos=0):
    """Times the reference CPU path (oracle/_ref) -- or the C restatement when
    the reference build is absent -- on the host cores: one warm-up token at
    start_pos, then up to n_max tokens (bounded to ~budget_s) at the positions
    after it -- the positions the GPU loop is timed at, so each step attends
    over as many cache rows (a step's cost does not depend on the rows'
    contents, so no prompt is ingested first).
    Returns (tokens/s, cores, kind, sample description)."""
    import numpy as np

    import oracle
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    if oracle.ref_available(cfg.ctx > 512):
        model, kind = oracle.RefModel(path, cfg.ctx), "reference"
    else:
        model, kind = oracle.OracleModel(path, cfg.ctx), "port"
    tok = synth_prompt(cfg)[0]
    t = time.perf_counter()
    logits = model.forward(tok, start_pos)
    t_warm = time.perf_counter() - t
    n = int(max(2, min(n_max, budget_s / max(t_warm, 1e-3), cfg.ctx - start_pos - 1)))
    t = time.perf_counter()
    for i in range(n):
        tok = int(np.argmax(logits))
        logits = model.forward(tok, start_pos + 1 + i)
    dt = time.perf_counter() - t
    model.close()
    sample = (f"{n} greedy decode tokens at positions {start_pos + 1}..{start_pos + n} (after 1 "
              f"warm-up token at position {start_pos}; the cache rows before it attended over "
              f"as at those positions) of the same GGUF, {cores} OpenMP threads, "
              f"{'reference C code built from the PhoneMap sources' if kind == 'reference' else 'C restatement of the reference'}")
    return n / dt, cores, kind, sample


def cpu_sample_run(logits, temperature, top_p, top_k, draws=20):
    """Times the reference's own ss_sample (tensor.c:363-451; oracle/_ref, or
    the C restatement when the reference build is absent) on the host: `draws`
    chained draws from one logits vector, one thread (ss_sample is serial).
    Returns (ms per draw, kind)."""
    import oracle
    if oracle.ref_available():
        fn, kind = oracle.ref_sample, "reference"
    else:
        fn, kind = (lambda x, t, p, k, s: oracle.sample(x, t, p, k, s, 0)), "port"
    state = 0x9E3779B97F4A7C15
    fn(logits, temperature, top_p, top_k, state)
    t = time.perf_counter()
    for _ in range(draws):
        _, state = fn(logits, temperature, top_p, top_k, state)
    return (time.perf_counter() - t) / draws * 1000.0, kind


def synth_prompt(cfg):
    from phonemap_b200 import synth
    return synth.prompt_tokens(cfg)


# ---------------------------------------------------------------- main paths

def share_from_rank0(pg, make):
    """Rank 0's value of make() on every rank (an object broadcast; make is
    called on rank 0 only) -- how the tensor-parallel group's NCCL id reaches
    every rank."""
    box = [make() if pg is None or pg.get_rank() == 0 else None]
    if pg is not None:
        pg.broadcast_object_list(box, src=0)
    return box[0]


def max_over_ranks(pg, x: float, device: str = "cuda") -> float:
    """The largest x over the ranks (every rank gets it): multi-GPU times are
    the slowest rank's."""
    if pg is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def workload(cfg, args, persistent=True):
    return {
        "workload": (f"{cfg.name}-shaped llama decoder, {'Q4_0' if cfg.wtype == 2 else 'Q8_0'} "
                     f"weights, greedy decode at batch 1 after a {cfg.prompt}-token prompt"),
        "weights": "Q4_0" if cfg.wtype == 2 else "Q8_0",
        "prompt_tokens": cfg.prompt,
        "decode_positions": [cfg.prompt + args.warmup, cfg.prompt + args.warmup + args.steps - 1],
        "batch": 1,
        "ctx": cfg.ctx,
        "l2": "inputs larger than L2 (weights streamed per step exceed the 126 MB L2)",
        "parallelism": ("single GPU" if args.gpus <= 1 else
                        f"dp{args.gpus} (independent replicas)" if args.replicas else
                        f"tp{args.gpus} (tensor parallel; "
                        + ("exchanges over NVLink peer memory inside the persistent step)" if persistent
                           else "NCCL all-reduces between the step's kernels)")),
        **({"hbm_budget_layers": budget_layers_of(cfg, args),
            "weights": f"{'Q4_0' if cfg.wtype == 2 else 'Q8_0'}, layers past the resident ones "
                       "copied from the host-mapped model file every step (layer streaming)"}
           if budget_layers_of(cfg, args) else {}),
    }


def batch_workload(cfg, args, world):
    P, W, K, B = cfg.prompt, args.warmup, args.steps, args.batch
    return {
        "workload": (f"{cfg.name}-shaped llama decoder, {'Q4_0' if cfg.wtype == 2 else 'Q8_0'} "
                     f"weights, {B} sequences decoded together (greedy) after {P}-token prompts each"),
        "batch": B, "prompt_tokens": P, "ctx": cfg.ctx,
        "decode_positions": [P + W, P + W + K - 1],
        "l2": "inputs larger than L2 (weights streamed per step exceed the 126 MB L2)",
        "parallelism": "single GPU" if world <= 1 else f"dp{world} (independent replicas)",
    }


def budget_layers_of(cfg, args):
    """HBM budget for the layers' weights, in layers (0: all resident)."""
    if args.hbm_budget_layers is not None:
        return args.hbm_budget_layers
    return 4 if cfg.name == "llama2-13b" else 0


def run_reference(args):
    world, rank, _, pg = dist_setup(args)
    if rank != 0:
        return 0
    from phonemap_b200 import configs, synth
    cfg = configs.get(args.config)
    path = synth.ensure_gguf(cfg)
    n_max = max(1, args.steps)
    B = max(1, args.batch)
    value, cores, kind, sample = cpu_reference_run(cfg, path, n_max, budget_s=90.0,
                                                   start_pos=cfg.prompt + args.warmup)
    if B > 1:  # the reference decodes one sequence at a time: B sequences cost B times one
        sample += f"; the reference has no batched decode, so {B} sequences take {B} times as long"
    line = {
        "metric": f"decode tokens/s (batch {B})", "value": round(value, 4), "unit": "tokens/s",
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / value, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init GGUF)",
        "config": batch_workload(cfg, args, args.gpus) if B > 1 else workload(cfg, args),
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": cores,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    world, rank, local, pg = dist_setup(args)
    import numpy as np
    import torch

    from phonemap_b200 import configs, runtime, synth
    cfg = configs.get(args.config)
    if rank == 0:
        path = synth.ensure_gguf(cfg)
    if pg:
        pg.barrier()
    path = synth.ensure_gguf(cfg)
    torch.cuda.set_device(local)
    flags = runtime.FLAG_MULTI_KERNEL if args.multi_kernel else 0
    tp = world if (world > 1 and not args.replicas) else 1
    budget_layers = budget_layers_of(cfg, args)
    budget = int(budget_layers * (cfg.layer_bytes() + 4096)) if budget_layers else 0
    if budget and tp > 1:
        raise SystemExit("layer streaming runs on one GPU (use --replicas with --gpus N)")
    if budget:
        m = runtime.CudaModel(path, cfg.ctx, device=local, flags=flags, hbm_budget_bytes=budget)
    elif tp > 1:
        nid = share_from_rank0(pg, runtime.tp_unique_id)
        m = runtime.CudaModel(path, cfg.ctx, device=local, flags=flags, tp_rank=rank, tp_size=tp,
                              tp_nccl_id=nid)
    else:
        m = runtime.CudaModel(path, cfg.ctx, device=local, flags=flags)
    seqs = world // tp  # sequences decoded concurrently by the whole job
    prompt = synth.prompt_tokens(cfg)
    P, W, K = len(prompt), args.warmup, args.steps
    if P + W + K + 1 > cfg.ctx:
        raise SystemExit("prompt + warmup + steps exceed the context")
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))

    # ---- device-resident decode loop (inputs already in HBM)
    first = m.prefill(prompt, 0)
    m.decode_begin(first, P)
    m.decode_steps(W)
    m.decode_read(P + 1, 1)
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.05)
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        t_w0 = time.perf_counter()
        ev0.record(stream)
        m.decode_steps(K)
        ev1.record(stream)
        ev1.synchronize()
        t_w1 = time.perf_counter()
        torch.cuda.synchronize()
        sampler.window = (t_w0, t_w1)
        time.sleep(0.02)
    ms = ev0.elapsed_time(ev1)
    ids = m.decode_read(P + 1, W + K)
    if pg:
        ms = max_over_ranks(pg, ms)
        pg.barrier()
    ms_per_step = ms / K
    value = seqs * K / (ms / 1000.0)
    stats = m.stats()

    # ---- end to end through the public C ABI with host buffers: per step the
    # token and position go host->device, the logits and argmax device->host
    e2e = None
    if not args.no_e2e:
        m.reset()
        logits = np.empty(m.vocab, np.float32)
        tok = m.prefill(prompt, 0)
        pos = P
        for _ in range(W):
            tok = m.forward(tok, pos, logits=logits)
            pos += 1
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(K):
            tok = m.forward(tok, pos, logits=logits)
            pos += 1
        dt = time.perf_counter() - t0
        dt = max_over_ranks(pg, dt)
        e2e = {"value": round(seqs * K / dt, 2), "unit": "tokens/s",
               "h2d_bytes_per_step": 4 + 8, "d2h_bytes_per_step": 4 * m.vocab + 4 + 4,
               "api": "ss_cuda_forward (host token in, host logits + argmax out, synchronous)"}

    # ---- sampled generation (ss_sample on the device between steps,
    # ss_cuda_decode_sample): K draws and K - 1 steps from the prompt's logits,
    # device-timed on the context's stream; then one draw alone
    sampled = None
    if tp == 1 and args.sample != "off":
        st, sp, sk = args.sample.split(",")
        st, sp, sk = float(st), float(sp), int(sk)
        m.reset()
        m.prefill(prompt, 0)
        m.decode_sample(P, min(W, 4) + 1, st, sp, sk, 0x9E3779B97F4A7C15)  # warm-up (sampler buffers)
        m.reset()
        first_logits = np.empty(m.vocab, np.float32)
        m.prefill(prompt, 0, logits=first_logits)
        torch.cuda.synchronize()
        ev0.record(stream)
        s_ids, _ = m.decode_sample(P, K, st, sp, sk, 0x9E3779B97F4A7C15)
        ev1.record(stream)
        ev1.synchronize()
        s_ms = ev0.elapsed_time(ev1)
        draw_ms = m.time_kernel("sample" if (st, sp, sk) == (0.7, 0.9, 40) else "sample_topp", 20)
        sampled = {"value": round(K / (s_ms / 1000.0), 2), "unit": "tokens/s",
                   "settings": {"temperature": st, "top_p": sp, "top_k": sk},
                   "ms_per_token": round(s_ms / K, 4), "ms_per_draw": round(draw_ms, 4),
                   "api": "ss_cuda_decode_sample (draws on the device, one CTA, the reference's "
                          "summation order)", "first_ids": s_ids[:8]}
        if rank == 0 and not args.no_cpu_baseline:
            cpu_ms, cpu_kind = cpu_sample_run(first_logits, st, sp, sk)
            sampled["cpu_baseline"] = {"ms_per_draw": round(cpu_ms, 4), "cores": 1, "kind": cpu_kind,
                                       "sample": "20 chained ss_sample draws from the prompt's logits"}

    # ---- roofline of the dominant kernel.  Persistent step: the one kernel
    # is the whole step; its algorithmic bytes are the step's (all weights at
    # the GGUF's bytes per weight + norms + one embedding row + the int8 K/V
    # read and append at the average timed position), its duration the CUDA-
    # event time per step above.  Multi-kernel step: the gate/up GEMV (2*ff*d
    # weights; this rank's ff/tp rows under tensor parallelism), timed live in
    # isolated back-to-back launches.  The step roofline of a tensor-parallel
    # group is the whole model's bytes per token against tp GPUs' bandwidth.
    peak, peak_kind = hbm_peak()
    step_bytes = cfg.token_bytes(P + W + (K - 1) / 2.0)
    step_gbs = step_bytes / (ms_per_step / 1000.0) / 1e9
    host_link = None
    if stats["streamed_bytes"]:
        # layer streaming: the step is bound by the host-to-device copies of the
        # streamed layers; their rate against a measured pinned-memory copy
        h2d = measure_h2d_gbs(local)
        got = stats["streamed_bytes"] / (ms_per_step / 1000.0) / 1e9
        host_link = {"bound": "host-link", "bytes_per_step": int(stats["streamed_bytes"]),
                     "achieved": round(got, 2), "peak": round(h2d, 2), "unit": "GB/s",
                     "frac": round(got / h2d, 4),
                     "peak_source": "measured here: 1 GiB pinned host-to-device cudaMemcpyAsync",
                     "resident_layers": stats["resident_layers"], "layers": cfg.n_layers,
                     "source": {1: "registered model mapping", 2: "pinned host copy",
                                3: "pageable memory"}.get(stats["stream_source"], "?")}
    if stats["persistent"]:
        # tensor parallelism: each rank's kernel streams its 1/tp of the bytes
        kernel_name = "decode_step_kernel (persistent: the whole decode step" + (
            f", one rank of {tp})" if tp > 1 else ")")
        k_bytes, k_ms = step_bytes / tp, ms_per_step
        achieved = k_bytes / (k_ms / 1000.0) / 1e9
        traffic = read_profile_traffic("decode_step", cfg.name) if tp == 1 else None
    else:
        kernel_name = "gate/up GEMV + RMSNorm + SwiGLU"
        bpw = 18 / 32 if cfg.wtype == 2 else 34 / 32
        ff_l = cfg.ffn // tp
        k_bytes = 2 * ff_l * cfg.d_model * bpw + cfg.d_model * 4 * 2 + ff_l * 4
        k_ms = m.time_kernel("gate_up", 3 * cfg.n_layers)
        achieved = k_bytes / (k_ms / 1000.0) / 1e9
        traffic = read_profile_traffic("gemv_gate_up", cfg.name)
    m.close()

    line = None
    if rank == 0:
        line = {
            "metric": "decode tokens/s (batch 1)", "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong" if tp > 1 else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init GGUF, N(0,0.02) quantized)",
            "config": workload(cfg, args, bool(stats["persistent"])),
            "roofline": {"bound": "hbm", "kernel": kernel_name,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "bytes_per_launch": int(k_bytes), "ms_per_launch": round(k_ms, 5),
                         "traffic": traffic},
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved": round(step_gbs, 1),
                              "frac": round(step_gbs / (tp * peak), 4), "unit": "GB/s",
                              "peak": round(tp * peak, 1), "peak_source": peak_kind,
                              "gpus_per_sequence": tp},
            "e2e": e2e,
            **({"sampled": sampled} if sampled else {}),
            "gpu_launches": int(stats["kernels_per_step"] * K),
            **({"host_link": host_link} if host_link else {}),
            "clocks": sampler.summary(),
            "step_impl": ("persistent single kernel" + (" (tensor-parallel: in-kernel peer-memory exchanges)"
                                                        if tp > 1 else "")
                          if stats["persistent"] else
                          "multi-kernel CUDA graph" + (" with NCCL all-reduces" if tp > 1 else "")),
            "pdl": bool(stats["pdl"]),
            "first_ids": ids[:8],
        }
        if world == 1 and not args.no_cpu_baseline:
            v, cores, kind, sample = cpu_reference_run(cfg, path, K, start_pos=P + W)
            line["cpu_baseline"] = {"value": round(v, 4), "unit": "tokens/s", "cores": cores,
                                    "kind": kind, "sample": sample}
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_ours_batch(args):
    """B sequences decoded together on each GPU through the many-token step
    (one pass of the tensor-core product per layer matrix for all B tokens).
    value: device-resident greedy loop (ss_cuda_decode_greedy_batch: tokens fed
    back on the device), B * steps / CUDA-event time; e2e: ss_cuda_forward with
    n_seq = B from host buffers, logits [B][vocab] and greedy tokens back every
    step.  With --gpus N each rank runs an independent replica (weak scaling)."""
    world, rank, local, pg = dist_setup(args)
    import numpy as np
    import torch

    from phonemap_b200 import configs, runtime, synth
    cfg = configs.get(args.config)
    B = args.batch
    if rank == 0:
        synth.ensure_gguf(cfg)
    if pg:
        pg.barrier()
    path = synth.ensure_gguf(cfg)
    torch.cuda.set_device(local)
    m = runtime.CudaModel(path, cfg.ctx, device=local, max_batch=B)
    P, W, K = cfg.prompt, args.warmup, args.steps
    if P + W + K + 1 > cfg.ctx:
        raise SystemExit("prompt + warmup + steps exceed the context")
    rng = np.random.default_rng(7)
    prompts = rng.integers(0, cfg.vocab, size=(B, P)).astype(np.int32)
    prompts[0] = np.asarray(synth.prompt_tokens(cfg), np.int32)[:P]
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))

    t0 = time.perf_counter()
    first = m.prefill_batch(prompts, 0)
    prefill_s = time.perf_counter() - t0
    warm = m.decode_greedy_batch(first, P, W)
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.05)
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        t_w0 = time.perf_counter()
        ev0.record(stream)
        ids = m.decode_greedy_batch(warm[-1], P + W, K)
        ev1.record(stream)
        ev1.synchronize()
        t_w1 = time.perf_counter()
        sampler.window = (t_w0, t_w1)
        time.sleep(0.02)
    ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(pg, ms)
    ms_per_step = ms / K
    value = world * B * K / (ms / 1000.0)
    stats = m.stats()

    e2e = None
    if not args.no_e2e:
        m.reset()
        logits = np.empty((B, m.vocab), np.float32)
        toks = m.prefill_batch(prompts, 0)
        pos = P
        for _ in range(W):
            toks = m.forward_batch(toks, pos, logits=logits)
            pos += 1
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(K):
            toks = m.forward_batch(toks, pos, logits=logits)
            pos += 1
        dt = max_over_ranks(pg, time.perf_counter() - t0)
        e2e = {"value": round(world * B * K / dt, 2), "unit": "tokens/s",
               "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B * m.vocab + 4 * B,
               "api": "ss_cuda_forward with n_seq = B (host tokens in, host logits [B][vocab] + "
                      "greedy tokens out, synchronous)"}

    # sampled: the same B sequences with a draw per sequence each step
    # (ss_cuda_decode_sample_batch), device-timed like the greedy loop
    sampled = None
    if args.sample != "off":
        st, sp, sk = args.sample.split(",")
        st, sp, sk = float(st), float(sp), int(sk)
        seeds = [0x9E3779B97F4A7C15 + 2 * i for i in range(B)]
        m.reset()
        first = m.prefill_batch(prompts, 0)
        warm, _ = m.decode_sample_batch(first, P, max(W, 1), st, sp, sk, seeds)
        torch.cuda.synchronize()
        ev0.record(stream)
        s_ids, _ = m.decode_sample_batch(warm[-1], P + max(W, 1), K, st, sp, sk, seeds)
        ev1.record(stream)
        ev1.synchronize()
        s_ms = max_over_ranks(pg, ev0.elapsed_time(ev1))
        sampled = {"value": round(world * B * K / (s_ms / 1000.0), 2), "unit": "tokens/s",
                   "settings": {"temperature": st, "top_p": sp, "top_k": sk},
                   "ms_per_step": round(s_ms / K, 4),
                   "api": "ss_cuda_decode_sample_batch (one draw per sequence on the device each step)",
                   "first_ids": s_ids[0].tolist()[:8]}

    # roofline: the tensor-core gate/up product at B tokens (the kernel alone,
    # cycling the layers so the weights stream from HBM); algorithmic bytes =
    # the matrix's GGUF bytes (weights + fp16 scales) + the activation pieces
    # (B x ff... fp16 hi/lo of d columns) + the fp32 outputs
    peak, peak_kind = hbm_peak()
    k_ms = m.time_kernel("product_gate_up", 3 * cfg.n_layers)
    bpw = 18 / 32 if cfg.wtype == 2 else 34 / 32
    k_bytes = 2 * cfg.ffn * cfg.d_model * bpw + B * cfg.d_model * 4 + B * 2 * cfg.ffn * 4
    achieved = k_bytes / (k_ms / 1000.0) / 1e9
    traffic = read_profile_traffic("qgemm", f"{cfg.name}-b{B}")
    # one step streams the weights once and each sequence's K/V rows (plus the
    # other sequences' embedding rows)
    avg = P + W + (K - 1) / 2.0
    kv_seq = cfg.n_layers * 2 * (cfg.kv_dim + 4) * (avg + 2)
    step_bytes = cfg.token_bytes(avg) + (B - 1) * (kv_seq + cfg.d_model * 4)
    step_gbs = step_bytes / (ms_per_step / 1000.0) / 1e9
    m.close()
    if rank == 0:
        line = {
            "metric": f"decode tokens/s (batch {B})", "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init GGUF, N(0,0.02) quantized; seeded prompts)",
            "config": batch_workload(cfg, args, world),
            "roofline": {"bound": "hbm", "kernel": "qgemm_kernel (gate/up, tcgen05 kind::f16, "
                                                   f"{B} tokens)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "bytes_per_launch": int(k_bytes), "ms_per_launch": round(k_ms, 5),
                         "traffic": traffic},
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved": round(step_gbs, 1),
                              "frac": round(step_gbs / peak, 4), "unit": "GB/s", "peak": peak,
                              "peak_source": peak_kind},
            "e2e": e2e,
            **({"sampled": sampled} if sampled else {}),
            "gpu_launches": int(stats["kernels_per_batched_step"] * K),
            "clocks": sampler.summary(),
            "step_impl": "many-token step: tensor-core product per matrix (CUDA graph per batch shape)",
            "prefill_s": round(prefill_s, 3),
            "first_ids": [int(v) for v in ids[:4, 0]],
        }
        if world == 1 and not args.no_cpu_baseline:
            v, cores, kind, sample = cpu_reference_run(cfg, path, K, start_pos=P + W)
            line["cpu_baseline"] = {"value": round(v, 4), "unit": "tokens/s", "cores": cores,
                                    "kind": kind, "sample": sample + "; the reference decodes one "
                                    "sequence at a time, so B sequences take B times as long"}
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def measure_h2d_gbs(device: int) -> float:
    """Pinned host-to-device copy bandwidth (1 GiB, 3 copies after a warm-up)."""
    import torch
    n = 1 << 30
    src = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(n, dtype=torch.uint8, device=f"cuda:{device}")
    s = torch.cuda.Stream(device=device)
    with torch.cuda.stream(s):
        dst.copy_(src, non_blocking=True)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        e1.record(s)
    e1.synchronize()
    gbs = 3 * n / (e0.elapsed_time(e1) / 1000.0) / 1e9
    del src, dst
    return gbs


def run_profile_kernel(args):
    """Times one kernel of the decode step in isolation (3 warm-up + --steps
    launches, cycling through the layers) and prints its bandwidth -- the small
    case the ncu captures in profiles/ are taken on."""
    from phonemap_b200 import configs, runtime, synth
    cfg = configs.get(args.config)
    path = synth.ensure_gguf(cfg)
    per_kernel = args.profile_kernel != "step"
    flags = runtime.FLAG_MULTI_KERNEL if (per_kernel or args.multi_kernel) else 0
    if args.profile_kernel.startswith("product_"):
        flags = 0
    m = runtime.CudaModel(path, cfg.ctx, device=0, flags=flags, max_batch=max(1, args.batch))
    if args.profile_kernel in ("attention", "step"):  # give it cached positions to attend over
        m.prefill(synth.prompt_tokens(cfg), 0)
    ms = m.time_kernel(args.profile_kernel, args.steps)
    nbytes = m.kernel_bytes(args.profile_kernel)
    print(json.dumps({"kernel": args.profile_kernel, "config": cfg.name, "launches": args.steps,
                      "ms_per_launch": round(ms, 5), "device_bytes": nbytes,
                      "GBps": round(nbytes / (ms / 1000.0) / 1e9, 1) if nbytes > 0 else None,
                      "stats": m.stats()}), flush=True)
    m.close()
    return 0


def main():
    args = parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.profile_kernel:
        return run_profile_kernel(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.batch > 1:
        return run_ours_batch(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
