"""CPU oracles for the SlipStream decode path -- TEST INFRASTRUCTURE ONLY.

Two implementations, both CPU:

* ``RefModel`` drives the reference's own C code (harrisonfar123/PhoneMap,
  ``SlipStream/src``), compiled by ``oracle/build_ref.py`` into
  ``oracle/_ref/libss_ref*.so``.
* ``OracleModel`` drives ``oracle/ss_oracle.c``, this repository's plain-C
  restatement of the same algorithm (each function cites the reference
  file:line it follows), compiled into ``oracle/_build/libss_oracle.so``.  It is
  pinned against ``RefModel`` bit for bit and against the golden fixtures in
  ``tests/golden/``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package; the product (``phonemap_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
BUILD_DIR = os.path.join(HERE, "_build")
ORACLE_LIB = os.path.join(BUILD_DIR, "libss_oracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(_i32p)


def build_oracle(force: bool = False) -> str:
    """Compile ss_oracle.c with gcc -O2 like the reference's own build.
    -ffp-contract=off keeps every product and sum of the reference order
    separately rounded; -mfma only makes the explicit fmaf() of the blocked
    order (sso_set_dot_order(1)) a hardware instruction."""
    src = os.path.join(HERE, "ss_oracle.c")
    hdr = os.path.join(HERE, "ss_oracle.h")
    if (force or not os.path.exists(ORACLE_LIB)
            or os.path.getmtime(ORACLE_LIB) < max(os.path.getmtime(src), os.path.getmtime(hdr))):
        os.makedirs(BUILD_DIR, exist_ok=True)
        subprocess.run(["gcc", "-std=gnu11", "-O2", "-mfma", "-ffp-contract=off", "-fopenmp",
                        "-fPIC", "-shared", src, "-o", ORACLE_LIB, "-lm"], check=True)
    return ORACLE_LIB


def ref_available(ctx8k: bool = False) -> bool:
    return os.path.exists(os.path.join(REF_DIR, "libss_ref_ctx8k.so" if ctx8k else "libss_ref.so"))


def build_ref() -> bool:
    """Build oracle/_ref from the reference tree when it is present."""
    r = subprocess.run(["python3", os.path.join(HERE, "build_ref.py")],
                       stdout=subprocess.DEVNULL)
    return r.returncode == 0


class _Model:
    """Common driver: prefill + greedy decode over a flat C API."""

    _lib: ctypes.CDLL
    _h: ctypes.c_void_p
    vocab: int

    def prefill(self, tokens, start_pos: int = 0) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.vocab, np.float32)
        if self._prefill(self._h, _ip(toks), len(toks), start_pos, _fp(out)) != 0:
            raise RuntimeError("prefill failed")
        return out

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        if self._forward(self._h, int(token), int(pos), _fp(out)) != 0:
            raise RuntimeError("forward failed")
        return out

    def greedy(self, prompt, n_steps: int, keep_logits=(), start_pos: int = 0) -> tuple[list[int], dict]:
        """Prefill then greedy decode, as engine.c:211-289 with temperature 0.
        The prompt's first token sits at `start_pos` (0 as in engine.c).

        Returns the generated IDs (the first comes from the prefill logits) and
        {step: logits} for the requested steps (step 0 = prefill logits)."""
        kept = {}
        logits = self.prefill(prompt, start_pos)
        ids = []
        pos = start_pos + len(prompt)
        for step in range(n_steps):
            if step in keep_logits:
                kept[step] = logits.copy()
            tok = int(np.argmax(logits))  # first maximum, as ss_argmax (tensor.c:318-328)
            ids.append(tok)
            if step + 1 < n_steps:
                logits = self.forward(tok, pos)
                pos += 1
        return ids, kept


class RefModel(_Model):
    """The reference C implementation (oracle/_ref)."""

    def __init__(self, gguf_path: str, ctx: int, ctx8k: bool | None = None, cuda_hook: bool = False):
        """cuda_hook: the integration build (libss_ref_cuda.so, the reference
        with the CUDA backend in its ss_matmul_dispatch); attach_cuda() hands
        it a context."""
        if ctx8k is None:
            ctx8k = ctx > 512
        name = "libss_ref_cuda.so" if cuda_hook else "libss_ref_ctx8k.so" if ctx8k else "libss_ref.so"
        lib = ctypes.CDLL(os.path.join(REF_DIR, name))
        if cuda_hook:
            lib.ssr_attach_cuda.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.ssr_load.restype = ctypes.c_void_p
        lib.ssr_load.argtypes = [ctypes.c_char_p, ctypes.c_uint32]
        for fn in ("ssr_free", "ssr_reset"):
            getattr(lib, fn).argtypes = [ctypes.c_void_p]
        lib.ssr_dims.argtypes = [ctypes.c_void_p, _i32p]
        lib.ssr_prefill.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p]
        lib.ssr_forward.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, _f32p]
        lib.ssr_embed.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, _f32p]
        lib.ssr_kv_row.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                   ctypes.c_void_p, ctypes.c_void_p, _f32p, _f32p]
        self._lib = lib
        self._h = ctypes.c_void_p(lib.ssr_load(gguf_path.encode(), ctx))
        if not self._h:
            raise RuntimeError(f"reference failed to load {gguf_path}")
        dims = np.zeros(8, np.int32)
        lib.ssr_dims(self._h, _ip(dims))
        (self.vocab, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads,
         self.head_dim, self.ffn, self.max_seq) = (int(v) for v in dims)
        self._prefill = lib.ssr_prefill
        self._forward = lib.ssr_forward

    def reset(self):
        self._lib.ssr_reset(self._h)

    def attach_cuda(self, cuda_ctx) -> None:
        """Give the hooked reference's scheduler a CUDA context (None detaches)."""
        self._lib.ssr_attach_cuda(self._h, cuda_ctx)

    def embed(self, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.hidden, np.float32)
        if self._lib.ssr_embed(self._h, _ip(toks), len(toks), _fp(out)) != 0:
            raise RuntimeError("embed failed")
        return out

    def kv_row(self, layer: int, pos: int):
        kvd = self.n_kv_heads * self.head_dim
        k = np.empty(kvd, np.int8)
        v = np.empty(kvd, np.int8)
        ks = ctypes.c_float()
        vs = ctypes.c_float()
        self._lib.ssr_kv_row(self._h, layer, pos, k.ctypes.data, v.ctypes.data,
                             ctypes.byref(ks), ctypes.byref(vs))
        return k, v, ks.value, vs.value

    def close(self):
        if self._h:
            self._lib.ssr_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_ops():
    """The reference's single ops (dequantize, dequant-matvec, rmsnorm, rope ...)."""
    lib = ctypes.CDLL(os.path.join(REF_DIR, "libss_ref.so"))
    lib.ssr_dequantize.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int32, ctypes.c_int32]
    lib.ssr_dequant_matvec.argtypes = [_f32p, ctypes.c_void_p, _f32p, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32]
    lib.ssr_matvec_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int32, ctypes.c_int32]
    lib.ssr_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int32, ctypes.c_float]
    lib.ssr_rope.argtypes = [_f32p, _f32p] + [ctypes.c_int32] * 5 + [ctypes.c_float]
    lib.ssr_softmax.argtypes = [_f32p, ctypes.c_int32]
    lib.ssr_argmax.argtypes = [_f32p, ctypes.c_int32]
    lib.ssr_argmax.restype = ctypes.c_int32
    lib.ssr_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.ssr_f16_to_f32.restype = ctypes.c_float
    return lib


class OracleModel(_Model):
    """This repository's C restatement (oracle/ss_oracle.c)."""

    def __init__(self, gguf_path: str, ctx: int, cap512: bool = False):
        lib = ctypes.CDLL(build_oracle())
        lib.sso_load.restype = ctypes.c_void_p
        lib.sso_load.argtypes = [ctypes.c_char_p, ctypes.c_uint32, ctypes.c_int]
        for fn in ("sso_free", "sso_reset"):
            getattr(lib, fn).argtypes = [ctypes.c_void_p]
        lib.sso_dims.argtypes = [ctypes.c_void_p, _i32p]
        lib.sso_prefill.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p]
        lib.sso_forward.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, _f32p]
        lib.sso_embed.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, _f32p]
        lib.sso_kv_row.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                   ctypes.c_void_p, ctypes.c_void_p, _f32p, _f32p]
        self._lib = lib
        self._h = ctypes.c_void_p(lib.sso_load(gguf_path.encode(), ctx, int(cap512)))
        if not self._h:
            raise RuntimeError(f"oracle failed to load {gguf_path}")
        dims = np.zeros(8, np.int32)
        lib.sso_dims(self._h, _ip(dims))
        (self.vocab, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads,
         self.head_dim, self.ffn, self.max_seq) = (int(v) for v in dims)
        self._prefill = lib.sso_prefill
        self._forward = lib.sso_forward
        lib.sso_set_dot_order.argtypes = [ctypes.c_void_p, ctypes.c_int]

    def set_dot_order(self, mode: int) -> None:
        """0: the reference's sequential sums; 1: GPU-shaped blocked order."""
        self._lib.sso_set_dot_order(self._h, int(mode))

    def reset(self):
        self._lib.sso_reset(self._h)

    def embed(self, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.hidden, np.float32)
        if self._lib.sso_embed(self._h, _ip(toks), len(toks), _fp(out)) != 0:
            raise RuntimeError("embed failed")
        return out

    def kv_row(self, layer: int, pos: int):
        kvd = self.n_kv_heads * self.head_dim
        k = np.empty(kvd, np.int8)
        v = np.empty(kvd, np.int8)
        ks = ctypes.c_float()
        vs = ctypes.c_float()
        self._lib.sso_kv_row(self._h, layer, pos, k.ctypes.data, v.ctypes.data,
                             ctypes.byref(ks), ctypes.byref(vs))
        return k, v, ks.value, vs.value

    def close(self):
        if self._h:
            self._lib.sso_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def oracle_ops():
    """Single ops of the restatement."""
    lib = ctypes.CDLL(build_oracle())
    lib.sso_dequantize.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int32, ctypes.c_int32]
    lib.sso_dequant_matvec.argtypes = [_f32p, ctypes.c_void_p, _f32p, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32]
    lib.sso_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int32, ctypes.c_float]
    lib.sso_rope.argtypes = [_f32p, _f32p] + [ctypes.c_int32] * 5 + [ctypes.c_float]
    lib.sso_kv_encode.argtypes = [_f32p, ctypes.c_void_p, _f32p, ctypes.c_int32]
    lib.sso_softmax.argtypes = [_f32p, ctypes.c_int32]
    lib.sso_argmax.argtypes = [_f32p, ctypes.c_int32]
    lib.sso_argmax.restype = ctypes.c_int32
    lib.sso_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.sso_f16_to_f32.restype = ctypes.c_float
    return lib


_u64p = ctypes.POINTER(ctypes.c_uint64)


def _sample_args(fn) -> None:
    fn.argtypes = [_f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_int32, _u64p]
    fn.restype = ctypes.c_int32


def sample(logits: np.ndarray, temperature: float, top_p: float, top_k: int, state: int,
           exp_mode: int = 0) -> tuple[int, int]:
    """ss_sample restated (oracle/ss_oracle.c): (token, new RNG state).
    exp_mode 0 is libm's expf, as the reference; 1 the GPU sampler's
    double-precision exponential."""
    lib = ctypes.CDLL(build_oracle())
    fn = lib.sso_sample
    fn.argtypes = [_f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_int32, _u64p,
                   ctypes.c_int]
    fn.restype = ctypes.c_int32
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    st = ctypes.c_uint64(state)
    tok = fn(_fp(lg), lg.size, temperature, top_p, int(top_k), ctypes.byref(st), int(exp_mode))
    return int(tok), int(st.value)


def exp_dd(x: np.ndarray) -> np.ndarray:
    """The GPU sampler's exponential, restated (sso_exp_dd)."""
    lib = ctypes.CDLL(build_oracle())
    lib.sso_exp_dd_array.argtypes = [_f32p, _f32p, ctypes.c_int32]
    xa = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(xa)
    lib.sso_exp_dd_array(_fp(xa), _fp(out), xa.size)
    return out


def ref_sample(logits: np.ndarray, temperature: float, top_p: float, top_k: int,
               state: int) -> tuple[int, int]:
    """The reference's own ss_sample (tensor.c:363-451, oracle/_ref build)."""
    lib = ctypes.CDLL(os.path.join(REF_DIR, "libss_ref.so"))
    _sample_args(lib.ss_sample)
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    st = ctypes.c_uint64(state)
    tok = lib.ss_sample(_fp(lg), lg.size, temperature, top_p, int(top_k), ctypes.byref(st))
    return int(tok), int(st.value)
