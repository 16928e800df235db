"""CPU simulation of the tensor-parallel sharding (tests/tp_sim.py): the
weights split exactly as the CUDA backend's upload splits them, each rank's
partial outputs summed in rank order, the int8 K/V scale taken over every
rank's maxima, and the token over every rank's best -- compared with the
unsharded model and with the reference's golden token IDs.  Runs as threads of
one process and as two gloo ranks (torch.distributed), no GPU."""
from __future__ import annotations

import os

import numpy as np
import pytest

from phonemap_b200 import configs, synth
from tests import tp_sim
from tests.conftest import load_golden, rel_err

STEPS = 6


def _golden_prompt(name):
    g = load_golden(name)
    return [int(t) for t in g["prompt"]], [int(t) for t in g["ids"]]


@pytest.mark.parametrize("name,tp", [("tiny", 2), ("tiny-mha", 2), ("tiny-mha", 4), ("tiny-q8", 2)])
def test_sharded_matches_whole_and_reference(name, tp):
    cfg = configs.get(name)
    path = synth.ensure_gguf(cfg)
    prompt, ref_ids = _golden_prompt(name)
    ids1, lg1 = tp_sim.run_local(path, cfg, 1, prompt, STEPS)
    idsn, lgn = tp_sim.run_local(path, cfg, tp, prompt, STEPS)
    assert ids1 == ref_ids[:STEPS]          # the restatement against the reference
    assert idsn == ids1                     # sharding changes no token
    for a, b in zip(lgn, lg1):
        assert rel_err(a, b) < 1e-4         # rank-order sums: fp32 rounding only
    g = load_golden(name)
    assert rel_err(lg1[0], g["logits"][0]) < 1e-4


def _gloo_rank(rank, world, path_cfg, prompt, out_dir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            init_method=f"file://{out_dir}/rdv")
    try:
        name = path_cfg
        cfg = configs.get(name)
        path = synth.ensure_gguf(cfg)
        w = tp_sim.dequantized(path)
        shard = tp_sim.Shard(w, tp_sim.model_dims(path, cfg), rank, world, 64)

        def allmax(x):
            t = torch.from_numpy(np.ascontiguousarray(x))
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.numpy()

        def allsum(x):
            parts = [torch.empty(x.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(x)))
            acc = parts[0].numpy().copy()
            for p in parts[1:]:
                acc = (acc + p.numpy()).astype(np.float32)
            return acc

        def allbest(k):
            # unsigned 64-bit order as signed: subtract 2^63 before, add it after
            t = torch.tensor([k - (1 << 63)], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return int(t.item()) + (1 << 63)

        ids, pos = [], 0
        for t in range(len(prompt) + STEPS - 1):
            tok = prompt[t] if t < len(prompt) else ids[-1]
            nxt, _ = shard.step(tok, pos, allmax, allsum, allbest)
            pos += 1
            if t >= len(prompt) - 1:
                ids.append(int(nxt))
        np.save(os.path.join(out_dir, f"ids{rank}.npy"), np.array(ids))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    """The same exchanges over torch.distributed gloo, one process per rank:
    both ranks produce the reference's token IDs."""
    import torch.multiprocessing as mp
    prompt, ref_ids = _golden_prompt("tiny")
    synth.ensure_gguf(configs.get("tiny"))
    mp.spawn(_gloo_rank, args=(2, "tiny", prompt, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert list(np.load(tmp_path / f"ids{r}.npy")) == ref_ids[:STEPS]
