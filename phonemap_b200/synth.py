"""Seeded synthetic GGUF models (benchmark and test inputs).

``ensure_gguf(cfg)`` returns the path of the GGUF file for a
``configs.ModelConfig``, writing it with the native writer
(``csrc/synth_gguf.c``) the first time.  Files are cached under
``$SS_GGUF_CACHE`` (default ``$TMPDIR/ss_gguf_cache``) by a hash of every
parameter that determines their bytes, so the same configuration yields the
same bytes on every host.
"""
from __future__ import annotations

import ctypes
import os
import tempfile

from . import build
from .configs import ModelConfig

WRITER_VERSION = 1


class _SynthConfig(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_uint32), ("d_model", ctypes.c_uint32),
        ("n_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
        ("vocab", ctypes.c_uint32), ("ctx", ctypes.c_uint32),
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("wtype", ctypes.c_int32), ("out_type", ctypes.c_int32),
        ("seed", ctypes.c_uint64), ("stddev", ctypes.c_float),
        ("norm_jitter", ctypes.c_float),
    ]


_lib = None


def _writer():
    global _lib
    if _lib is None:
        path = build.SYNTH_LIB
        if not os.path.exists(path):
            path = build.build_synth()
        _lib = ctypes.CDLL(path)
        _lib.ss_synth_write_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(_SynthConfig)]
        _lib.ss_synth_write_gguf.restype = ctypes.c_int
    return _lib


def cache_dir() -> str:
    d = os.environ.get("SS_GGUF_CACHE") or os.path.join(tempfile.gettempdir(), "ss_gguf_cache")
    os.makedirs(d, exist_ok=True)
    return d


def gguf_path(cfg: ModelConfig) -> str:
    return os.path.join(cache_dir(), f"{cfg.name}-v{WRITER_VERSION}-{cfg.model_key()}.gguf")


def write_gguf(cfg: ModelConfig, path: str) -> None:
    c = _SynthConfig(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                     cfg.ffn, cfg.vocab, cfg.ctx, cfg.rope_theta, cfg.rms_eps, cfg.wtype,
                     cfg.wtype, cfg.seed, cfg.stddev, cfg.norm_jitter)
    rc = _writer().ss_synth_write_gguf(path.encode(), ctypes.byref(c))
    if rc != 0:
        raise RuntimeError(f"ss_synth_write_gguf({path}) failed with {rc}")


def ensure_gguf(cfg: ModelConfig) -> str:
    path = gguf_path(cfg)
    if not os.path.exists(path):
        fd, tmp = tempfile.mkstemp(dir=os.path.dirname(path), suffix=".part")
        os.close(fd)
        try:
            write_gguf(cfg, tmp)
            os.replace(tmp, path)
        finally:
            if os.path.exists(tmp):
                os.unlink(tmp)
    return path


def prompt_tokens(cfg: ModelConfig, n: int | None = None, seq: int = 0) -> list[int]:
    """Seeded uniform token IDs in [0, vocab) (numpy default_rng)."""
    import numpy as np
    rng = np.random.default_rng(cfg.seed * 1000 + 17 + seq)
    return [int(t) for t in rng.integers(0, cfg.vocab, size=n or cfg.prompt)]
