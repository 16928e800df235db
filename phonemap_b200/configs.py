"""Model shapes and workloads of the five benchmark configurations.

Each entry is a seeded random-init llama decoder written as GGUF (see
``phonemap_b200.synth``).  Shapes follow the configuration list the benchmark
is quoted on; the small ``tiny*`` shapes exist only so that the CPU oracle
finishes in seconds inside the parity tests.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json

Q4_0 = 2
Q8_0 = 8
TYPE_NAMES = {Q4_0: "Q4_0", Q8_0: "Q8_0", 0: "F32"}


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    ctx: int
    wtype: int = Q4_0
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    seed: int = 1234
    stddev: float = 0.02
    norm_jitter: float = 0.0
    # workload
    prompt: int = 32
    decode: int = 128
    batch: int = 1

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def model_key(self) -> str:
        """Hash of everything that determines the GGUF bytes."""
        keys = ("n_layers", "d_model", "n_heads", "n_kv_heads", "ffn", "vocab", "ctx",
                "wtype", "rope_theta", "rms_eps", "seed", "stddev", "norm_jitter")
        blob = json.dumps({k: getattr(self, k) for k in keys}, sort_keys=True)
        return hashlib.sha1(blob.encode()).hexdigest()[:12]

    def layer_bytes(self) -> int:
        """GGUF bytes of one layer's seven quantized matrices."""
        bpw = 18 / 32 if self.wtype == Q4_0 else 34 / 32
        d, qd, kvd, ff = self.d_model, self.n_heads * self.head_dim, self.kv_dim, self.ffn
        return int((d * qd + 2 * d * kvd + qd * d + 3 * d * ff) * bpw)

    def weight_bytes(self) -> int:
        """Quantized bytes streamed per decode token (all layers + lm_head)."""
        bpw = 18 / 32 if self.wtype == Q4_0 else 34 / 32
        return int(self.layer_bytes() * self.n_layers + self.vocab * self.d_model * bpw)

    def token_bytes(self, pos: float) -> float:
        """Algorithmic HBM bytes for one decode token at position ``pos``.

        Quantized weights + fp32 norm weights + one fp32 embedding row + the
        int8 K/V cache read over positions 0..pos (int8 values + one fp32 scale
        per row) + the K/V append, per layer.
        """
        d, L = self.d_model, self.n_layers
        norms = (2 * L + 1) * d * 4
        embed = d * 4
        kv_read = L * 2 * (self.kv_dim + 4) * (pos + 1)
        kv_write = L * 2 * (self.kv_dim + 4)
        return self.weight_bytes() + norms + embed + kv_read + kv_write


CONFIGS: dict[str, ModelConfig] = {
    # TinyLlama-1.1B shape, the reference's own CPU-runnable case
    "tinyllama": ModelConfig("tinyllama", 22, 2048, 32, 4, 5632, 32000, 512,
                             prompt=32, decode=128),
    # the headline -- Llama-2-7B shape, Q4_0, batch 1
    "llama2-7b": ModelConfig("llama2-7b", 32, 4096, 32, 32, 11008, 32000, 2048,
                             prompt=128, decode=256),
    # Llama-3-8B shape, Q8_0, GQA 32/8, theta 5e5
    "llama3-8b": ModelConfig("llama3-8b", 32, 4096, 32, 8, 14336, 128256, 4096,
                             wtype=Q8_0, rope_theta=500000.0, prompt=512, decode=256),
    # Llama-2-13B shape, streamed with 4 resident layers
    "llama2-13b": ModelConfig("llama2-13b", 40, 5120, 40, 40, 13824, 32000, 1024,
                              prompt=32, decode=128),
    # Llama-2-70B shape, GQA 64/8
    "llama2-70b": ModelConfig("llama2-70b", 80, 8192, 64, 8, 28672, 32000, 2048,
                              prompt=256, decode=128),
    # profiling: Llama-2-7B layer shapes, 2 layers (< 1 GB on the device), for
    # small-case ncu captures of the same kernels
    "llama2-7b-2l": ModelConfig("llama2-7b-2l", 2, 4096, 32, 32, 11008, 32000, 2048,
                                prompt=128, decode=256),
    # Llama-2-70B layer shapes (d 8192, GQA 64/8, FFN 28672), 4 layers: every
    # kernel instantiation of configs[4] in a 3 GB file, for the parity suite
    "llama2-70b-4l": ModelConfig("llama2-70b-4l", 4, 8192, 64, 8, 28672, 32000, 2048,
                                 prompt=256, decode=128),
    # Llama-3-8B layer shapes, 2 layers: the Q8_0 / 128256-vocab kernels in a
    # small file (profiling and quick checks)
    "llama3-8b-2l": ModelConfig("llama3-8b-2l", 2, 4096, 32, 8, 14336, 128256, 4096,
                                wtype=Q8_0, rope_theta=500000.0, prompt=512, decode=256),
    # parity-test shapes (oracle finishes in seconds)
    "tiny": ModelConfig("tiny", 2, 256, 8, 2, 512, 512, 128, norm_jitter=0.1,
                        prompt=8, decode=24, seed=7),
    "tiny-mha": ModelConfig("tiny-mha", 3, 512, 4, 4, 1024, 1000, 128, norm_jitter=0.1,
                            prompt=5, decode=20, seed=11),
    "tiny-q8": ModelConfig("tiny-q8", 2, 256, 8, 2, 768, 600, 128, wtype=Q8_0,
                           norm_jitter=0.1, rope_theta=500000.0, prompt=6, decode=20,
                           seed=13),
}


def get(name: str) -> ModelConfig:
    try:
        return CONFIGS[name]
    except KeyError as e:
        raise KeyError(f"unknown config {name!r}; known: {sorted(CONFIGS)}") from e
