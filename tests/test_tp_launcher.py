"""Host-side logic of the tensor-parallel launcher (phonemap_b200/tp.py), on
CPU: the group's ranks are spawned processes; a rank that fails reports its
traceback and the parent ends the whole group within its timeout instead of
leaving the other ranks waiting."""
from __future__ import annotations

import time

import pytest

from phonemap_b200 import tp


def test_failed_rank_ends_the_group():
    t0 = time.time()
    with pytest.raises(RuntimeError) as e:
        # no such model file: rank 0 fails while the other waits for its NCCL id
        tp.greedy("/nonexistent/model.gguf", 64, [1, 2, 3], 4, 2, timeout=120)
    assert "tensor-parallel group failed" in str(e.value)
    assert "rank" in str(e.value)
    assert time.time() - t0 < 120
