"""The synthetic GGUF writer: deterministic bytes, metadata the reference loader
reads, tensor shapes [ne0 = cols, ne1 = rows]."""
from __future__ import annotations

import dataclasses
import os
import struct

from phonemap_b200 import configs, synth


def test_deterministic(tmp_path):
    cfg = dataclasses.replace(configs.get("tiny"), name="det")
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    synth.write_gguf(cfg, str(a))
    synth.write_gguf(cfg, str(b))
    assert a.read_bytes() == b.read_bytes()
    c = tmp_path / "c.gguf"
    synth.write_gguf(dataclasses.replace(cfg, seed=cfg.seed + 1), str(c))
    assert a.read_bytes() != c.read_bytes()


def test_header_fields():
    cfg = configs.get("tiny")
    data = open(synth.ensure_gguf(cfg), "rb").read(1 << 16)
    magic, version, n_t, n_kv = struct.unpack_from("<IIQQ", data)
    assert magic == 0x46554747 and version == 3
    assert n_t == 3 + 9 * cfg.n_layers and n_kv == 12


def test_weight_bytes_formula():
    cfg = configs.get("llama2-7b")
    # 32 layers x (4 x 4096^2 + 3 x 4096 x 11008) + lm_head, Q4_0 = 18/32 B per weight
    assert cfg.weight_bytes() == int((32 * (4 * 4096 ** 2 + 3 * 4096 * 11008) + 32000 * 4096) * 18 / 32)
    assert abs(cfg.token_bytes(256) / 1e9 - 3.785) < 0.02
