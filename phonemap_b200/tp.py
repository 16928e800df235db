"""Tensor-parallel decode in one process per GPU, for callers that are not
already launched one rank per GPU (torchrun launches bench.py that way).

`greedy(path, ctx, prompt, steps, tp)` spawns `tp` ranks; rank r opens the
model on GPU r as rank r of an NCCL group (the library's own communicator; the
id travels from rank 0 through a queue) and decodes the same sequence.  Every
rank takes the same collective steps in the same order; rank 0 returns the
results.  A rank that fails reports its error and the parent ends the group,
so a failed initialisation never leaves the others waiting past `timeout`.
"""
from __future__ import annotations

import multiprocessing as mp
import queue
import traceback


def _sampled(m, prompt, steps, sample):
    """Sampled decode two ways on one context: ss_cuda_decode_sample (draws
    and steps on the device), and a host loop of ss_cuda_sample draws from the
    device logits and ss_cuda_forward steps that also copies each step's logits
    and the RNG state before each draw out (for a check of every draw)."""
    import numpy as np
    t, p, k, seed = sample
    m.reset()
    m.prefill(prompt, 0)
    dev_ids, dev_state = m.decode_sample(len(prompt), steps, t, p, k, seed)
    m.reset()
    buf = np.empty(m.vocab, np.float32)
    m.prefill(prompt, 0, logits=buf)
    ids, states, logits, s = [], [seed], [buf.copy()], seed
    for i in range(steps):
        tok, s = m.sample(t, p, k, s)
        ids.append(tok)
        states.append(s)
        if i + 1 < steps:
            m.forward(tok, len(prompt) + i, logits=buf)
            logits.append(buf.copy())
    return {"dev_ids": dev_ids, "dev_state": dev_state, "ids": ids, "states": states,
            "logits": np.stack(logits)}


def _rank_main(rank, tp, path, ctx, prompt, steps, teacher, flags, kv_at, id_q, out_q, sample=None):
    try:
        import numpy as np
        import torch  # noqa: F401  (loads the process's NCCL before the library resolves it)

        from phonemap_b200 import runtime
        if rank == 0:
            nid = runtime.tp_unique_id()
            for _ in range(tp - 1):
                id_q.put(nid)
        else:
            nid = id_q.get(timeout=120)
        m = runtime.CudaModel(path, ctx, device=rank, flags=flags, tp_rank=rank, tp_size=tp,
                              tp_nccl_id=nid)
        logits = np.empty((steps, m.vocab), np.float32)
        buf = np.empty(m.vocab, np.float32)
        ids = [m.prefill(prompt, 0, logits=buf)]
        logits[0] = buf
        pos = len(prompt)
        for s in range(1, steps):
            tok = teacher[s - 1] if teacher is not None else ids[-1]
            ids.append(m.forward(tok, pos, logits=buf))
            logits[s] = buf
            pos += 1
        kv = m.kv_row(*kv_at)
        # the device-resident loop (no host round trip per token) over the same sequence
        m.reset()
        first = m.prefill(prompt, 0)
        loop_ids = [first] + list(m.decode_greedy(first, len(prompt), steps - 1))
        stats = m.stats()
        sampled = _sampled(m, prompt, steps, sample) if sample is not None else None
        m.close()
        if rank == 0:
            res = {"ids": ids, "logits": logits, "loop_ids": loop_ids, "kv_row0": kv, "stats": stats,
                   "sampled": sampled}
        else:  # every rank's draws, to check that all ranks drew the same tokens
            res = {"sampled_ids": None if sampled is None else (sampled["dev_ids"], sampled["ids"])}
        out_q.put((rank, None, res))
    except BaseException:
        out_q.put((rank, traceback.format_exc(), None))


def greedy(path: str, ctx: int, prompt, steps: int, tp: int, teacher=None, flags: int = 0,
           kv_at=(0, 0), timeout: float = 600.0, sample=None) -> dict:
    """Greedy decode of `steps` tokens after `prompt` over a `tp`-GPU group.
    teacher: tokens fed at steps 1.. instead of the model's own argmax.
    Returns rank 0's ids, logits [steps][vocab], the device-loop ids, rank 0's
    int8 K/V row (its kv heads) at kv_at = (layer, pos) and its stats.
    sample = (temperature, top_p, top_k, seed): also `steps` sampled tokens
    after the prompt (rank 0's under "sampled", see _sampled; every other
    rank's tokens under "sampled_ids_other")."""
    ctx_mp = mp.get_context("spawn")
    id_q, out_q = ctx_mp.Queue(), ctx_mp.Queue()
    prompt = [int(t) for t in prompt]
    teacher = None if teacher is None else [int(t) for t in teacher]
    procs = [ctx_mp.Process(target=_rank_main,
                            args=(r, tp, path, ctx, prompt, steps, teacher, flags, tuple(kv_at), id_q,
                                  out_q, None if sample is None else tuple(sample)))
             for r in range(tp)]
    for p in procs:
        p.start()
    result, errors, others = None, [], []
    try:
        for _ in range(tp):
            try:
                rank, err, res = out_q.get(timeout=timeout)
            except queue.Empty:
                errors.append(f"no answer within {timeout:.0f} s")
                break
            if err:
                errors.append(f"rank {rank}: {err}")
                break
            if rank == 0:
                result = res
            else:
                others.append(res["sampled_ids"])
    finally:
        for p in procs:
            p.join(timeout=30 if not errors else 5)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
    if errors or result is None:
        raise RuntimeError("tensor-parallel group failed: " + "; ".join(errors or ["no result"]))
    result["sampled_ids_other"] = others
    return result
