#!/usr/bin/env python3
"""Build the reference SlipStream CPU path into ``oracle/_ref/`` (TEST INFRASTRUCTURE).

The reference (harrisonfar123/PhoneMap, ``SlipStream/``) is C written for Apple
platforms.  Its hot path -- ``ss_scheduler_forward`` / ``ss_scheduler_prefill``
(SlipStream/src/core/layer_scheduler.c:571-803) and everything under them --
compiles with gcc after four mechanical adaptations, applied to a *temporary
copy* of the sources (nothing from the reference is ever written into this
repository; only the built ``.so`` and test binaries land in ``oracle/_ref/``):

1. ``<Accelerate/Accelerate.h>``, ``<dispatch/dispatch.h>`` and
   ``<sys/sysctl.h>`` resolve to the stand-ins in ``oracle/shims/``.
2. Every ``dispatch_apply(N, q, ^(size_t i){ ... });`` (quantize.c:475,
   layer_scheduler.c:424) becomes an OpenMP parallel-for with the same blocking
   semantics, and every ``dispatch_async(q, ^{ ... });``
   (layer_scheduler.c:612,726,849, bodies are no-op prefetches) becomes an
   inline block.
3. ``model->metal`` (engine.c:112, a field that exists only with SS_HAS_METAL)
   becomes NULL.
4. The two literal 512-position caps (layer_scheduler.c:202 and the stack
   ``scores[512]`` at :430) become ``SS_REF_MAX_SEQ``.  ``libss_ref.so`` is
   built with 512 (faithful); ``libss_ref_ctx8k.so`` with 8192 (the "patched
   oracle" needed by configurations that run past 512 positions).

A fifth build, ``libss_ref_cuda.so``, is the reference with this
repository's CUDA backend plugged in the way a maintainer would (INTEGRATION.md
section 4): ``ss_scheduler_t`` gains a ``cuda_ctx`` next to its ``metal_ctx``
(layer_scheduler.h:80) and ``ss_matmul_dispatch`` (layer_scheduler.c:248-279)
gains an ``#ifdef SS_HAS_CUDA`` branch before its CPU fallback that calls
``ss_cuda_matvec_q4_0`` / ``_q8_0`` / ``ss_cuda_matvec`` (include/
slipstream_cuda.h) -- the reference's own scheduler, with every projection
served by the GPU.  It links against ``phonemap_b200/lib/libslipstream_cuda.so``
(built first) and is only made when that library exists.

Usage: ``python oracle/build_ref.py [--src <SlipStream dir>] [--out oracle/_ref]``
Exit status 0 when built, 2 when the reference tree is absent.
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def default_src() -> str:
    """The reference's SlipStream directory: $SS_REFERENCE_SRC, else
    ``<reference_path>/SlipStream`` from the repository's BASELINE.json."""
    env = os.environ.get("SS_REFERENCE_SRC")
    if env:
        return env
    try:
        import json
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            return os.path.join(json.load(f)["reference_path"], "SlipStream")
    except (OSError, KeyError, ValueError):
        return ""

CORE_SOURCES = [
    "src/core/engine.c",
    "src/core/gguf_loader.c",
    "src/core/layer_scheduler.c",
    "src/core/tensor.c",
    "src/core/quantize.c",
    "src/core/tokenizer.c",
    "src/utils/memory.c",
    "src/utils/thread_pool.c",
    "src/utils/profiler.c",
    "src/backends/cpu_neon.c",
]

_APPLY = re.compile(
    r"dispatch_apply\s*\(\s*(?P<n>[^,]+?)\s*,\s*dispatch_get_global_queue\s*\([^)]*\)\s*,"
    r"\s*\^\s*\(\s*size_t\s+(?P<var>\w+)\s*\)\s*\{"
)
_ASYNC = re.compile(
    r"dispatch_async\s*\(\s*dispatch_get_global_queue\s*\([^)]*\)\s*,\s*\^\s*\{"
)


def _match_brace(text: str, open_idx: int) -> int:
    """Index of the '}' matching text[open_idx] == '{' (skips comments/strings)."""
    depth = 0
    i = open_idx
    n = len(text)
    while i < n:
        c = text[i]
        if text.startswith("//", i):
            i = text.index("\n", i)
            continue
        if text.startswith("/*", i):
            i = text.index("*/", i) + 2
            continue
        if c in "\"'":
            j = i + 1
            while text[j] != c:
                j += 2 if text[j] == "\\" else 1
            i = j + 1
            continue
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return i
        i += 1
    raise ValueError("unbalanced block")


def _close_call(text: str, brace_idx: int) -> int:
    """After the block's '}', consume ')' and ';' and return the index past them."""
    j = brace_idx + 1
    while text[j].isspace():
        j += 1
    if text[j] != ")":
        raise ValueError("expected ')' after block")
    j += 1
    while text[j].isspace():
        j += 1
    if text[j] != ";":
        raise ValueError("expected ';' after block call")
    return j + 1


def rewrite_blocks(text: str) -> tuple[str, int]:
    """Rewrite Apple-blocks dispatch calls; returns (new_text, count)."""
    count = 0
    while True:
        m_apply = _APPLY.search(text)
        m_async = _ASYNC.search(text)
        cands = [m for m in (m_apply, m_async) if m]
        if not cands:
            return text, count
        m = min(cands, key=lambda mm: mm.start())
        open_idx = m.end() - 1
        close_idx = _match_brace(text, open_idx)
        end = _close_call(text, close_idx)
        body = text[open_idx + 1:close_idx]
        if m is m_apply:
            var, n = m.group("var"), m.group("n")
            head = (f'_Pragma("omp parallel for schedule(static)") '
                    f"for (size_t {var} = 0; {var} < (size_t)({n}); {var}++) {{")
        else:
            head = "{"
        text = text[:m.start()] + head + body + "}" + text[end:]
        count += 1


def prepare_tree(src: str, dst: str) -> None:
    for sub in ("src", "include"):
        shutil.copytree(os.path.join(src, sub), os.path.join(dst, sub))
    sched = os.path.join(dst, "src/core/layer_scheduler.c")
    quant = os.path.join(dst, "src/core/quantize.c")
    engine = os.path.join(dst, "src/core/engine.c")
    for path, expect in ((sched, 4), (quant, 1)):
        with open(path) as f:
            text = f.read()
        text, n = rewrite_blocks(text)
        if n != expect:
            raise RuntimeError(f"{path}: rewrote {n} dispatch blocks, expected {expect}")
        if path == sched:
            caps = [("if (max_seq > 512) max_seq = 512;",
                     "if (max_seq > SS_REF_MAX_SEQ) max_seq = SS_REF_MAX_SEQ;"),
                    ("float scores[512];", "float scores[SS_REF_MAX_SEQ];")]
            for old, new in caps:
                if text.count(old) != 1:
                    raise RuntimeError(f"512-cap pattern not found once: {old}")
                text = text.replace(old, new)
        with open(path, "w") as f:
            f.write(text)
    with open(engine) as f:
        text = f.read()
    text = text.replace("model->metal", "((void *)0)")
    with open(engine, "w") as f:
        f.write(text)


CUDA_BRANCH = """#ifdef SS_HAS_CUDA
    if (sched->cuda_ctx && ss_cuda_should_use_gpu(rows, cols)) {
        bool cuda_ok = false;
        if (type == GGML_TYPE_Q4_0)
            cuda_ok = ss_cuda_matvec_q4_0((ss_cuda_ctx_t *)sched->cuda_ctx, out, mat, vec, rows, cols);
        else if (type == GGML_TYPE_Q8_0)
            cuda_ok = ss_cuda_matvec_q8_0((ss_cuda_ctx_t *)sched->cuda_ctx, out, mat, vec, rows, cols);
        else if (type == GGML_TYPE_Q4_K)
            cuda_ok = ss_cuda_matvec_q4_K((ss_cuda_ctx_t *)sched->cuda_ctx, out, mat, vec, rows, cols);
        else if (type == GGML_TYPE_F32)
            cuda_ok = ss_cuda_matvec((ss_cuda_ctx_t *)sched->cuda_ctx, out, (const float *)mat, vec, rows, cols);
        if (cuda_ok) return;
    }
#endif

"""


def add_cuda_hook(tree: str) -> None:
    """The integration a maintainer adds, applied
    to the temporary copy: the context field and the dispatch branch."""
    hdr = os.path.join(tree, "src/core/layer_scheduler.h")
    with open(hdr) as f:
        text = f.read()
    anchor = "void             *metal_ctx;"
    if text.count(anchor) != 1:
        raise RuntimeError("metal_ctx field not found once in layer_scheduler.h")
    text = text.replace(anchor, anchor + "\n    void             *cuda_ctx;   /* ss_cuda_ctx_t (SS_HAS_CUDA) */")
    with open(hdr, "w") as f:
        f.write(text)
    sched = os.path.join(tree, "src/core/layer_scheduler.c")
    with open(sched) as f:
        text = f.read()
    anchor = "    // Fallback: execute on CPU NEON natively."
    if text.count(anchor) != 1:
        raise RuntimeError("CPU fallback anchor not found once in layer_scheduler.c")
    text = text.replace(anchor, CUDA_BRANCH + anchor)
    text = "#ifdef SS_HAS_CUDA\n#include \"slipstream_cuda.h\"\n#endif\n" + text
    with open(sched, "w") as f:
        f.write(text)


def build(src: str, out: str, cc: str = "gcc") -> list[str]:
    os.makedirs(out, exist_ok=True)
    built = []
    with tempfile.TemporaryDirectory(prefix="ss_ref_") as tmp:
        prepare_tree(src, tmp)
        inc = ["-I", os.path.join(HERE, "shims"), "-I", os.path.join(tmp, "include"),
               "-I", os.path.join(tmp, "src")]
        srcs = [os.path.join(tmp, s) for s in CORE_SOURCES]
        # -O2 as the reference's CMakeLists; no -march, so gcc emits no FMA and
        # every product/sum is rounded separately, as in the C source.
        flags = ["-std=gnu11", "-O2", "-fopenmp", "-fPIC", "-w"]
        for name, cap in (("libss_ref.so", 512), ("libss_ref_ctx8k.so", 8192)):
            target = os.path.join(out, name)
            cmd = [cc, *flags, f"-DSS_REF_MAX_SEQ={cap}", "-shared", *inc, *srcs,
                   os.path.join(HERE, "ref_driver.c"), "-o", target, "-lm"]
            subprocess.run(cmd, check=True)
            built.append(target)
        # the reference with the CUDA backend in its dispatch (needs the built library)
        repo = os.path.dirname(HERE)
        cuda_lib = os.path.join(repo, "phonemap_b200", "lib", "libslipstream_cuda.so")
        if os.path.exists(cuda_lib):
            hooked = os.path.join(tmp, "hooked")
            prepare_tree(src, hooked)
            add_cuda_hook(hooked)
            hinc = ["-I", os.path.join(HERE, "shims"), "-I", os.path.join(repo, "include"),
                    "-I", os.path.join(hooked, "include"), "-I", os.path.join(hooked, "src")]
            target = os.path.join(out, "libss_ref_cuda.so")
            rpath = os.path.relpath(os.path.dirname(cuda_lib), out)
            cmd = [cc, *flags, "-DSS_REF_MAX_SEQ=8192", "-DSS_HAS_CUDA", "-shared", *hinc,
                   *[os.path.join(hooked, x) for x in CORE_SOURCES], os.path.join(HERE, "ref_driver.c"),
                   "-o", target, "-L", os.path.dirname(cuda_lib), "-lslipstream_cuda",
                   f"-Wl,-rpath,$ORIGIN/{rpath}", "-lm"]
            subprocess.run(cmd, check=True)
            built.append(target)
        # the reference's own unit tests, linked against the same objects
        for test in ("test_quantize", "test_tensor_ops", "test_gguf_loader",
                     "test_layer_scheduler"):
            tsrc = os.path.join(src, "tests", test + ".c")
            if not os.path.exists(tsrc):
                continue
            target = os.path.join(out, test)
            cmd = [cc, *flags, "-DSS_REF_MAX_SEQ=512", *inc, tsrc, *srcs, "-o",
                   target, "-lm"]
            subprocess.run(cmd, check=True)
            built.append(target)
    return built


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=default_src())
    ap.add_argument("--out", default=os.path.join(HERE, "_ref"))
    args = ap.parse_args()
    if not os.path.isdir(os.path.join(args.src, "src", "core")):
        print(f"reference tree not found at {args.src}; nothing built", file=sys.stderr)
        return 2
    for path in build(args.src, args.out):
        print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
