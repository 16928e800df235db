"""Python binding of the CUDA backend's C ABI (include/slipstream_cuda.h).

``CudaModel`` mirrors the reference's scheduler entry points
(``ss_scheduler_forward`` / ``ss_scheduler_prefill`` / ``ss_scheduler_reset``,
SlipStream/src/core/layer_scheduler.h:107-132) and the Metal-shaped op-level
calls (``ss_metal_matvec_q4_0`` ..., SlipStream/src/backends/metal_backend.h:
27-70) one to one.  There is no CPU fallback: if the native library is missing
or the GPU call fails, these functions raise.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)

Q4_0, Q8_0, F32, Q4_K = 2, 8, 0, 12

# every symbol include/slipstream_cuda.h declares
EXPORTED = [
    "ss_cuda_default_options", "ss_cuda_init", "ss_cuda_init_file", "ss_cuda_free",
    "ss_cuda_last_error", "ss_cuda_abi_version", "ss_cuda_model_dims", "ss_cuda_stats",
    "ss_cuda_should_use_gpu", "ss_cuda_matvec", "ss_cuda_matvec_q4_0", "ss_cuda_matvec_q8_0",
    "ss_cuda_begin_batch", "ss_cuda_end_batch", "ss_cuda_scheduler_forward",
    "ss_cuda_scheduler_prefill", "ss_cuda_scheduler_reset", "ss_cuda_forward",
    "ss_cuda_prefill", "ss_cuda_decode_greedy", "ss_cuda_decode_begin", "ss_cuda_decode_steps",
    "ss_cuda_decode_read", "ss_cuda_stream", "ss_cuda_reset", "ss_cuda_cancel",
    "ss_cuda_dequantize_tensor", "ss_cuda_dequantize", "ss_cuda_kv_row",
    "ss_cuda_time_kernel", "ss_cuda_kernel_bytes", "ss_cuda_argmax_noalloc",
    "ss_cuda_step_trace", "ss_cuda_tp_unique_id", "ss_cuda_test_fail_next_step",
    "ss_cuda_matmul_batch", "ss_cuda_prefill_batch", "ss_cuda_decode_greedy_batch",
    "ss_cuda_embed", "ss_cuda_scheduler_embed", "ss_cuda_sample_logits", "ss_cuda_sample",
    "ss_cuda_decode_sample", "ss_cuda_decode_sample_batch", "ss_cuda_matvec_q4_K",
]


class SSCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class Options(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("device", ctypes.c_int32),
        ("context_size", ctypes.c_uint32), ("max_batch", ctypes.c_uint32),
        ("hbm_budget_bytes", ctypes.c_uint64), ("flags", ctypes.c_uint32),
        ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32),
        ("tp_nccl_id", ctypes.c_uint8 * 128),
    ]


FLAG_NO_PDL = 1
FLAG_NO_GRAPH = 2
FLAG_MULTI_KERNEL = 4
FLAG_TRACE = 8
FLAG_STEP_PREFILL = 16

_lib = None


def library_path() -> str:
    return build.CUDA_LIB


def load_library() -> ctypes.CDLL:
    """Load libslipstream_cuda.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.exists(path):
        raise ImportError(f"CUDA backend not built: {path} is missing "
                          "(run `python -m phonemap_b200.build`)")
    lib = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    lib.ss_cuda_default_options.argtypes = [ctypes.POINTER(Options)]
    lib.ss_cuda_init.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(Options)]
    lib.ss_cuda_init.restype = vp
    lib.ss_cuda_init_file.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options)]
    lib.ss_cuda_init_file.restype = vp
    lib.ss_cuda_free.argtypes = [vp]
    lib.ss_cuda_last_error.restype = ctypes.c_char_p
    lib.ss_cuda_model_dims.argtypes = [vp, _i32p]
    lib.ss_cuda_stats.argtypes = [vp, _i64p, ctypes.c_int32]
    lib.ss_cuda_should_use_gpu.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.ss_cuda_should_use_gpu.restype = ctypes.c_bool
    for fn in ("ss_cuda_matvec", "ss_cuda_matvec_q4_0", "ss_cuda_matvec_q8_0", "ss_cuda_matvec_q4_K"):
        getattr(lib, fn).argtypes = [vp, _f32p, vp, _f32p, ctypes.c_int32, ctypes.c_int32]
        getattr(lib, fn).restype = ctypes.c_bool
    for fn in ("ss_cuda_begin_batch", "ss_cuda_end_batch", "ss_cuda_reset",
               "ss_cuda_scheduler_reset", "ss_cuda_cancel"):
        getattr(lib, fn).argtypes = [vp]
    lib.ss_cuda_scheduler_forward.argtypes = [vp, ctypes.c_int32, ctypes.c_int32]
    lib.ss_cuda_scheduler_forward.restype = _f32p
    lib.ss_cuda_scheduler_prefill.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32]
    lib.ss_cuda_scheduler_prefill.restype = _f32p
    lib.ss_cuda_forward.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p, _i32p]
    lib.ss_cuda_prefill.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p]
    lib.ss_cuda_prefill_batch.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          _f32p, _i32p]
    lib.ss_cuda_decode_greedy_batch.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int32, _i32p]
    lib.ss_cuda_embed.argtypes = [vp, _i32p, ctypes.c_int32, _f32p]
    lib.ss_cuda_scheduler_embed.argtypes = [vp, _i32p, ctypes.c_int32]
    lib.ss_cuda_scheduler_embed.restype = ctypes.POINTER(ctypes.c_float)
    lib.ss_cuda_decode_greedy.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _i32p]
    lib.ss_cuda_decode_begin.argtypes = [vp, ctypes.c_int32, ctypes.c_int32]
    lib.ss_cuda_decode_steps.argtypes = [vp, ctypes.c_int32]
    lib.ss_cuda_decode_read.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, _i32p]
    lib.ss_cuda_stream.argtypes = [vp]
    lib.ss_cuda_stream.restype = vp
    lib.ss_cuda_dequantize_tensor.argtypes = [vp, ctypes.c_char_p, _f32p, ctypes.c_int64]
    lib.ss_cuda_dequantize.argtypes = [ctypes.c_int32, vp, ctypes.c_int64, _f32p]
    lib.ss_cuda_kv_row.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, vp, vp, _f32p, _f32p]
    lib.ss_cuda_time_kernel.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, _f32p]
    lib.ss_cuda_kernel_bytes.argtypes = [vp, ctypes.c_int32]
    lib.ss_cuda_kernel_bytes.restype = ctypes.c_int64
    lib.ss_cuda_matmul_batch.argtypes = [vp, ctypes.c_char_p, _f32p, ctypes.c_int32, _f32p]
    lib.ss_cuda_test_fail_next_step.argtypes = [vp, ctypes.c_int32]
    lib.ss_cuda_argmax_noalloc.argtypes = [vp, ctypes.c_int32, vp, vp]
    lib.ss_cuda_step_trace.argtypes = [vp, _i64p, ctypes.c_int64]
    lib.ss_cuda_tp_unique_id.argtypes = [vp]
    u64p = ctypes.POINTER(ctypes.c_uint64)
    fl, i32 = ctypes.c_float, ctypes.c_int32
    lib.ss_cuda_sample_logits.argtypes = [vp, _f32p, i32, fl, fl, i32, u64p, _i32p]
    lib.ss_cuda_sample.argtypes = [vp, fl, fl, i32, u64p, _i32p]
    lib.ss_cuda_decode_sample.argtypes = [vp, i32, i32, fl, fl, i32, u64p, _i32p]
    lib.ss_cuda_decode_sample_batch.argtypes = [vp, _i32p, i32, i32, i32, fl, fl, i32, u64p, _i32p]
    _lib = lib
    return lib


def _check(rc: int) -> int:
    if rc < 0:
        raise SSCudaError(rc, load_library().ss_cuda_last_error().decode())
    return rc


def _f(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _i(a: np.ndarray):
    return a.ctypes.data_as(_i32p)


def default_options(**kw) -> Options:
    o = Options()
    load_library().ss_cuda_default_options(ctypes.byref(o))
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def tp_unique_id() -> bytes:
    """An NCCL unique id for a tensor-parallel group (call on rank 0)."""
    buf = (ctypes.c_uint8 * 128)()
    _check(load_library().ss_cuda_tp_unique_id(buf))
    return bytes(buf)


class CudaModel:
    """One decode context on one GPU (one sequence, or up to max_batch)."""

    def __init__(self, gguf_path: str | None, context_size: int = 0, device: int = -1,
                 flags: int = 0, tp_rank: int = 0, tp_size: int = 1, tp_nccl_id: bytes = b"",
                 hbm_budget_bytes: int = 0, max_batch: int = 1):
        """tp_size > 1: this process is rank tp_rank of a tensor-parallel group
        whose NCCL id (tp_unique_id() on rank 0) is tp_nccl_id.
        hbm_budget_bytes > 0: HBM for the layers' weights; layers beyond it are
        streamed from the model file every step (layer streaming).
        max_batch > 1: sequences 0..max_batch-1 each keep a KV cache and decode
        together through forward_batch / prefill_batch."""
        lib = load_library()
        self._lib = lib
        opts = default_options(context_size=context_size, device=device, flags=flags,
                               tp_rank=tp_rank, tp_size=tp_size,
                               hbm_budget_bytes=int(hbm_budget_bytes), max_batch=int(max_batch))
        if tp_size > 1:
            if len(tp_nccl_id) != 128:
                raise ValueError("tp_nccl_id must be the 128 bytes of tp_unique_id()")
            ctypes.memmove(opts.tp_nccl_id, tp_nccl_id, 128)
        if gguf_path is None:
            h = lib.ss_cuda_init(None, 0, ctypes.byref(opts))
        else:
            h = lib.ss_cuda_init_file(gguf_path.encode(), ctypes.byref(opts))
        if not h:
            raise SSCudaError(-7, lib.ss_cuda_last_error().decode())
        self._h = ctypes.c_void_p(h)
        self.tp_rank, self.tp_size = (tp_rank, tp_size) if tp_size > 1 else (0, 1)
        if gguf_path is not None:
            dims = np.zeros(12, np.int32)
            _check(lib.ss_cuda_model_dims(self._h, _i(dims)))
            (self.vocab, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads,
             self.head_dim, self.ffn, self.ctx, self.rope_dim, self.wtype, self.max_batch,
             self.device) = (int(v) for v in dims)

    # ---- scheduler-level twins
    def scheduler_forward(self, token: int, pos: int) -> np.ndarray:
        p = self._lib.ss_cuda_scheduler_forward(self._h, int(token), int(pos))
        if not p:
            raise SSCudaError(-7, self._lib.ss_cuda_last_error().decode())
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def scheduler_prefill(self, tokens, start_pos: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        p = self._lib.ss_cuda_scheduler_prefill(self._h, _i(t), len(t), int(start_pos))
        if not p:
            raise SSCudaError(-7, self._lib.ss_cuda_last_error().decode())
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def scheduler_embed(self, tokens) -> np.ndarray:
        """ss_scheduler_embed's twin: a malloc'd vector, copied and freed here."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = self._lib.ss_cuda_scheduler_embed(self._h, _i(t), len(t))
        if not p:
            raise SSCudaError(-7, self._lib.ss_cuda_last_error().decode())
        out = np.ctypeslib.as_array(p, shape=(self.hidden,)).copy()
        ctypes.CDLL(None).free(ctypes.cast(p, ctypes.c_void_p))
        return out

    def reset(self) -> None:
        self._lib.ss_cuda_reset(self._h)

    def cancel(self) -> None:
        self._lib.ss_cuda_cancel(self._h)

    # ---- coarse entry points
    def forward(self, token: int, pos: int, logits: np.ndarray | None = None) -> int:
        t = np.array([token], np.int32)
        am = np.zeros(1, np.int32)
        lp = _f(logits) if logits is not None else None
        _check(self._lib.ss_cuda_forward(self._h, _i(t), 1, int(pos), lp, _i(am)))
        return int(am[0])

    def prefill(self, tokens, start_pos: int = 0, logits: np.ndarray | None = None) -> int:
        t = np.ascontiguousarray(tokens, np.int32)
        lp = _f(logits) if logits is not None else None
        return _check(self._lib.ss_cuda_prefill(self._h, _i(t), len(t), int(start_pos), lp))

    def forward_batch(self, tokens, pos: int, logits: np.ndarray | None = None) -> list[int]:
        """One step of sequences 0..len(tokens)-1 at position pos; greedy tokens.
        logits: optional float32 [len(tokens), vocab] output."""
        t = np.ascontiguousarray(tokens, np.int32)
        am = np.zeros(len(t), np.int32)
        if logits is not None and (logits.dtype != np.float32 or logits.size < len(t) * self.vocab
                                   or not logits.flags.c_contiguous):
            raise ValueError("logits must be contiguous float32 [n_seq, vocab]")
        lp = _f(logits) if logits is not None else None
        _check(self._lib.ss_cuda_forward(self._h, _i(t), len(t), int(pos), lp, _i(am)))
        return [int(v) for v in am]

    def prefill_batch(self, prompts, start_pos: int = 0,
                      logits: np.ndarray | None = None) -> list[int]:
        """Prompts [n_seq, n] of sequences 0..n_seq-1; greedy next token of each."""
        t = np.ascontiguousarray(prompts, np.int32)
        if t.ndim != 2:
            raise ValueError("prompts must be [n_seq, n]")
        am = np.zeros(t.shape[0], np.int32)
        if logits is not None and (logits.dtype != np.float32 or logits.size < t.shape[0] * self.vocab
                                   or not logits.flags.c_contiguous):
            raise ValueError("logits must be contiguous float32 [n_seq, vocab]")
        lp = _f(logits) if logits is not None else None
        _check(self._lib.ss_cuda_prefill_batch(self._h, _i(t), t.shape[0], t.shape[1], int(start_pos),
                                               lp, _i(am)))
        return [int(v) for v in am]

    def embed(self, tokens) -> np.ndarray:
        """Mean-pooled, L2-normalised final hidden state of the tokens
        (ss_scheduler_embed, positions 0..n-1)."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.hidden, np.float32)
        _check(self._lib.ss_cuda_embed(self._h, _i(t), len(t), _f(out)))
        return out

    def decode_greedy_batch(self, tokens, start_pos: int, n_steps: int) -> np.ndarray:
        """Greedy decode of sequences 0..len(tokens)-1 together, fed back on the
        device; returns int32 [n_steps, n_seq] (positions start_pos+1 ..)."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros((n_steps, len(t)), np.int32)
        _check(self._lib.ss_cuda_decode_greedy_batch(self._h, _i(t), len(t), int(start_pos),
                                                     int(n_steps), _i(out)))
        return out

    def decode_greedy(self, token: int, start_pos: int, n_steps: int) -> list[int]:
        out = np.zeros(n_steps, np.int32)
        _check(self._lib.ss_cuda_decode_greedy(self._h, int(token), int(start_pos), int(n_steps),
                                               _i(out)))
        return [int(v) for v in out]

    def decode_begin(self, token: int, pos: int) -> None:
        _check(self._lib.ss_cuda_decode_begin(self._h, int(token), int(pos)))

    def decode_steps(self, n: int) -> None:
        _check(self._lib.ss_cuda_decode_steps(self._h, int(n)))

    def decode_read(self, first_pos: int, n: int) -> list[int]:
        out = np.zeros(n, np.int32)
        _check(self._lib.ss_cuda_decode_read(self._h, int(first_pos), int(n), _i(out)))
        return [int(v) for v in out]

    # ---- sampling on the device (ss_sample, tensor.c:363-451)
    def sample_logits(self, logits, temperature: float, top_p: float = 1.0, top_k: int = 0,
                      state: int = 0) -> tuple[int, int]:
        """ss_sample over host logits: (token, RNG state after the draw)."""
        lg = np.ascontiguousarray(logits, np.float32)
        st = ctypes.c_uint64(int(state))
        tok = ctypes.c_int32(-1)
        _check(self._lib.ss_cuda_sample_logits(self._h, _f(lg), lg.size, float(temperature),
                                               float(top_p), int(top_k), ctypes.byref(st),
                                               ctypes.byref(tok)))
        return int(tok.value), int(st.value)

    def sample(self, temperature: float, top_p: float = 1.0, top_k: int = 0,
               state: int = 0) -> tuple[int, int]:
        """ss_sample over the last step's logits (on the device)."""
        st = ctypes.c_uint64(int(state))
        tok = ctypes.c_int32(-1)
        _check(self._lib.ss_cuda_sample(self._h, float(temperature), float(top_p), int(top_k),
                                        ctypes.byref(st), ctypes.byref(tok)))
        return int(tok.value), int(st.value)

    def decode_sample(self, start_pos: int, n_tokens: int, temperature: float, top_p: float = 1.0,
                      top_k: int = 0, state: int = 0) -> tuple[list[int], int]:
        """ss_generate's loop on the device: n_tokens draws, the first from the
        current logits, each next one after a decode step of the previous draw
        at start_pos, start_pos + 1, ...  Returns (tokens, RNG state)."""
        out = np.zeros(n_tokens, np.int32)
        st = ctypes.c_uint64(int(state))
        _check(self._lib.ss_cuda_decode_sample(self._h, int(start_pos), int(n_tokens),
                                               float(temperature), float(top_p), int(top_k),
                                               ctypes.byref(st), _i(out)))
        return [int(v) for v in out], int(st.value)

    def decode_sample_batch(self, tokens, start_pos: int, n_steps: int, temperature: float,
                            top_p: float = 1.0, top_k: int = 0,
                            states=None) -> tuple[np.ndarray, list[int]]:
        """Sequences 0..len(tokens)-1 decoded together with a draw per sequence
        each step (its own RNG state); returns (int32 [n_steps, n_seq] tokens of
        positions start_pos+1 .., the RNG states afterwards)."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros((n_steps, len(t)), np.int32)
        st = np.array(states if states is not None else [0] * len(t), np.uint64)
        _check(self._lib.ss_cuda_decode_sample_batch(
            self._h, _i(t), len(t), int(start_pos), int(n_steps), float(temperature), float(top_p),
            int(top_k), st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), _i(out)))
        return out, [int(v) for v in st]

    def greedy(self, prompt, n_steps: int) -> list[int]:
        """Prefill + greedy decode; same convention as oracle._Model.greedy."""
        first = self.prefill(prompt, 0)
        if n_steps <= 1:
            return [first][:n_steps]
        return [first] + self.decode_greedy(first, len(prompt), n_steps - 1)

    def matmul_batch(self, name: str, x: np.ndarray, rows: int) -> np.ndarray:
        """out[t] = W(name) . x[t] for the rows of x ([n_tokens][cols]) on the
        tensor cores (ss_cuda_matmul_batch)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], rows), np.float32)
        _check(self._lib.ss_cuda_matmul_batch(self._h, name.encode(), _f(x), x.shape[0], _f(out)))
        return out

    def test_fail_next_step(self, phase: int) -> None:
        """Test aid: the next persistent step withholds one weight copy and
        reports an error after its shortened waits run out."""
        _check(self._lib.ss_cuda_test_fail_next_step(self._h, int(phase)))

    def stream(self) -> int:
        return int(self._lib.ss_cuda_stream(self._h) or 0)

    def stats(self) -> dict:
        v = np.zeros(17, np.int64)
        _check(self._lib.ss_cuda_stats(self._h, v.ctypes.data_as(_i64p), 17))
        keys = ("kernels_per_step", "weight_bytes", "kv_bytes", "attn_splits", "pdl",
                "steps_run", "qkv_ctas", "down_ctas", "persistent", "ring_slots",
                "resident_layers", "streamed_bytes", "layer_bytes", "stream_source",
                "kernel_arch", "kernels_per_batched_step", "matvecs_run")
        return {k: int(x) for k, x in zip(keys, v)}

    KERNELS = {"qkv": 0, "attention": 1, "o": 2, "gate_up": 3, "down": 4, "lm_head": 5, "step": 6,
               "product_gate_up": 7, "product_qkv_l2": 8, "sample": 9, "sample_topp": 10}

    def time_kernel(self, which: str, iters: int) -> float:
        """Average ms per isolated launch of one step kernel (clobbers state)."""
        ms = np.zeros(1, np.float32)
        _check(self._lib.ss_cuda_time_kernel(self._h, self.KERNELS[which], int(iters), _f(ms)))
        return float(ms[0])

    def step_trace(self) -> np.ndarray:
        """Timeline of the last persistent step, [phase][cta][event] global-timer
        ns (context created with FLAG_TRACE; see ss_cuda_step_trace)."""
        st = self.stats()
        n = (2 + 5 * self.n_layers) * st["qkv_ctas"] * 8
        out = np.zeros(n, np.int64)
        _check(self._lib.ss_cuda_step_trace(self._h, out.ctypes.data_as(_i64p), n))
        return out.reshape(2 + 5 * self.n_layers, st["qkv_ctas"], 8)

    def kernel_bytes(self, which: str) -> int:
        return int(self._lib.ss_cuda_kernel_bytes(self._h, self.KERNELS[which]))

    # ---- inspection
    def dequantize_tensor(self, name: str, rows: int, cols: int) -> np.ndarray:
        out = np.empty(rows * cols, np.float32)
        _check(self._lib.ss_cuda_dequantize_tensor(self._h, name.encode(), _f(out), out.size))
        return out.reshape(rows, cols)

    def kv_row(self, layer: int, pos: int):
        """int8 K/V row of one position (this rank's kv heads under tensor
        parallelism) and its two scales."""
        kvd = self.n_kv_heads // self.tp_size * self.head_dim
        k = np.empty(kvd, np.int8)
        v = np.empty(kvd, np.int8)
        ks = np.zeros(1, np.float32)
        vs = np.zeros(1, np.float32)
        _check(self._lib.ss_cuda_kv_row(self._h, layer, pos, k.ctypes.data, v.ctypes.data,
                                        _f(ks), _f(vs)))
        return k, v, float(ks[0]), float(vs[0])

    # ---- op-level twins of the Metal calls
    def matvec(self, w_bytes: np.ndarray, x: np.ndarray, rows: int, cols: int, wtype: int) -> np.ndarray:
        out = np.empty(rows, np.float32)
        xx = np.ascontiguousarray(x, np.float32)
        fn = {Q4_0: self._lib.ss_cuda_matvec_q4_0, Q8_0: self._lib.ss_cuda_matvec_q8_0,
              Q4_K: self._lib.ss_cuda_matvec_q4_K, F32: self._lib.ss_cuda_matvec}[wtype]
        if not fn(self._h, _f(out), w_bytes.ctypes.data, _f(xx), rows, cols):
            raise SSCudaError(-7, self._lib.ss_cuda_last_error().decode())
        return out

    def begin_batch(self) -> None:
        self._lib.ss_cuda_begin_batch(self._h)

    def end_batch(self) -> None:
        self._lib.ss_cuda_end_batch(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.ss_cuda_free(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def argmax_noalloc(d_values: int, n: int, d_index: int, stream: int = 0) -> None:
    """ss_cuda_argmax_noalloc on device pointers (asynchronous on `stream`)."""
    _check(load_library().ss_cuda_argmax_noalloc(ctypes.c_void_p(d_values), int(n),
                                                  ctypes.c_void_p(d_index),
                                                  ctypes.c_void_p(stream or None)))


def dequantize_blocks(wtype: int, blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(load_library().ss_cuda_dequantize(wtype, blocks.ctypes.data, n, _f(out)))
    return out
