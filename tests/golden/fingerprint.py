"""Cheap fingerprint of a GGUF file: SHA-1 over its size plus 4 KiB sampled at
every 8 MiB and the final 4 KiB.  Used to check that a regenerated synthetic
model is byte-identical to the one the golden fixtures were made from."""
from __future__ import annotations

import hashlib
import os


def gguf_fingerprint(path: str) -> bytes:
    size = os.path.getsize(path)
    h = hashlib.sha1(str(size).encode())
    with open(path, "rb") as f:
        for off in list(range(0, size, 8 << 20)) + [max(0, size - 4096)]:
            f.seek(off)
            h.update(f.read(4096))
    return h.digest()
