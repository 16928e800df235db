"""The rank plumbing bench.py uses under torchrun, on CPU with the gloo backend
and two ranks: the tensor-parallel NCCL id made on rank 0 reaches every rank
unchanged, and a multi-rank time is the slowest rank's on every rank."""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import socket
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        import torch.distributed as dist

        import bench
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        made = []

        def make():
            made.append(rank)
            return bytes(range(128))
        nid = bench.share_from_rank0(dist, make)
        slowest = bench.max_over_ranks(dist, 1.5 * (rank + 1), device="cpu")
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, None, (nid, slowest, made)))
    except BaseException as e:  # report, never hang the parent
        q.put((rank, repr(e), None))


def test_rank0_id_and_max_over_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict()
        for _ in range(2):
            rank, err, val = q.get(timeout=120)
            assert err is None, f"rank {rank}: {err}"
            res[rank] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in (0, 1):
        nid, slowest, made = res[rank]
        assert nid == bytes(range(128))
        assert slowest == 3.0
        assert made == ([0] if rank == 0 else [])
