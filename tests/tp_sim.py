"""CPU simulation of the tensor-parallel sharding -- TEST INFRASTRUCTURE.

A numpy restatement of one llama decode step of SlipStream's CPU path
(SlipStream/src/core/layer_scheduler.c:291-567 per layer, :571-679 per token)
on fp32 weights dequantised by the oracle (bit-identical to the reference's
ss_dequantize), run either whole or as one rank of a tensor-parallel group with
the sharding the CUDA backend's upload applies (ss_cuda_api.cu, upload_matrix
calls in load_model):

* Q / K / V rows by heads: rank r keeps q heads [r nh/tp, (r+1) nh/tp) and kv
  heads [r nkv/tp, (r+1) nkv/tp) (GQA groups stay on one rank);
* O by the matching q-head columns, down by the matching FFN columns (both
  row-parallel: each rank's partial output, rank 0's carrying the residual,
  summed over ranks in rank order);
* gate / up by FFN rows; the lm_head by vocabulary rows [r V/tp, (r+1) V/tp);
* the int8 K/V scale of a position is the maximum of every rank's |k| / |v|
  maxima -- the reference's scale covers the whole kv_dim
  (layer_scheduler.c:101-111), so a rank holding some kv heads needs the
  others' maxima to produce the same int8 values;
* the greedy token is the maximum over ranks of the packed (value, index)
  (first maximum wins, as ss_argmax, tensor.c:318-328).

The exchanges are callables, so the same code runs in one process (a loop over
simulated ranks) or as real gloo ranks (tests/test_tp_sim.py).
"""
from __future__ import annotations

import ctypes

import numpy as np

import oracle
from tests.golden.crafted import tensor_table

_BLOCK = {2: 18, 8: 34}


def dequantized(path: str) -> dict:
    """{tensor name: fp32 array [rows, cols] (or 1-D for vectors)}."""
    ops = oracle.oracle_ops()
    out = {}
    for name, (off, ttype, dims) in tensor_table(path).items():
        cols = int(dims[0])
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        n = rows * cols
        if ttype == 0:
            a = np.fromfile(path, np.float32, count=n, offset=off)
        else:
            raw = np.fromfile(path, np.uint8, count=n // 32 * _BLOCK[ttype], offset=off)
            a = np.empty(n, np.float32)
            ops.sso_dequantize(raw.ctypes.data, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n,
                               ttype)
        out[name] = a.reshape(rows, cols) if len(dims) > 1 else a
    return out


def rmsnorm(x, w, eps):
    """cpu_neon.c:109-115: x * (1 / sqrtf(sum x^2 / n + eps)) * w."""
    ss = np.float32(np.dot(x.astype(np.float64), x))
    scale = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(x.size) + np.float32(eps)))
    return (x * scale * w).astype(np.float32)


def rope(vec, nheads, hd, rope_dim, pos, theta):
    """Non-NeoX RoPE (tensor.c:249-274) on `nheads` heads of `vec`."""
    v = vec.reshape(nheads, hd).copy()
    for i in range(0, rope_dim, 2):
        freq = np.float32(1.0) / np.float32(np.power(np.float32(theta), np.float32(i) / np.float32(rope_dim)))
        ang = np.float32(pos) * freq
        c, s = np.float32(np.cos(ang)), np.float32(np.sin(ang))
        a, b = v[:, i].copy(), v[:, i + 1].copy()
        v[:, i] = a * c - b * s
        v[:, i + 1] = a * s + b * c
    return v.reshape(-1)


def pack_argmax(v: float, idx: int) -> int:
    """The unsigned-max key of (value, index) whose maximum is ss_argmax's index."""
    if v != v:
        key = 0xFFFFFFFF if idx == 0 else 0
    else:
        b = int(np.array([0.0 if v == 0 else v], np.float32).view(np.uint32)[0])
        key = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (key << 32) | (0x7FFFFFFF - idx)


class Shard:
    """One rank's weights and KV cache (rank 0 of 1 = the whole model)."""

    def __init__(self, w: dict, dims: dict, rank: int = 0, tp: int = 1, ctx: int = 64):
        self.d, self.L, self.nh, self.nkv = dims["d"], dims["L"], dims["nh"], dims["nkv"]
        self.hd, self.ff, self.V = dims["hd"], dims["ff"], dims["V"]
        self.eps, self.theta = dims["eps"], dims["theta"]
        self.rank, self.tp = rank, tp
        nh, nkv, ff, hd = self.nh // tp, self.nkv // tp, self.ff // tp, self.hd
        self.nh_l, self.nkv_l, self.ff_l = nh, nkv, ff
        qd, kvd = nh * hd, nkv * hd
        self.Vl = self.V // tp
        r = rank
        self.embd = w["token_embd.weight"]
        self.out_norm = w["output_norm.weight"]
        self.head = w["output.weight"][r * self.Vl:(r + 1) * self.Vl]
        self.layers = []
        for l in range(self.L):
            p = f"blk.{l}."
            self.layers.append(dict(
                an=w[p + "attn_norm.weight"], fn=w[p + "ffn_norm.weight"],
                wq=w[p + "attn_q.weight"][r * qd:(r + 1) * qd],
                wk=w[p + "attn_k.weight"][r * kvd:(r + 1) * kvd],
                wv=w[p + "attn_v.weight"][r * kvd:(r + 1) * kvd],
                wo=w[p + "attn_output.weight"][:, r * qd:(r + 1) * qd],
                wg=w[p + "ffn_gate.weight"][r * ff:(r + 1) * ff],
                wu=w[p + "ffn_up.weight"][r * ff:(r + 1) * ff],
                wd=w[p + "ffn_down.weight"][:, r * ff:(r + 1) * ff]))
        self.kc = np.zeros((self.L, ctx, kvd), np.int8)
        self.vc = np.zeros((self.L, ctx, kvd), np.int8)
        self.ks = np.zeros((self.L, ctx), np.float32)
        self.vs = np.zeros((self.L, ctx), np.float32)

    def step(self, token: int, pos: int, allmax, allsum, allbest):
        """One decode token.  allmax(x) -> elementwise max over ranks;
        allsum(x) -> sum over ranks in rank order; allbest(k) -> max over ranks.
        Returns (token, this rank's logits)."""
        hd, G = self.hd, self.nh // self.nkv
        h = self.embd[token].astype(np.float32).copy()
        for l, ly in enumerate(self.layers):
            xn = rmsnorm(h, ly["an"], self.eps)
            q = (ly["wq"] @ xn).astype(np.float32)
            k = (ly["wk"] @ xn).astype(np.float32)
            v = (ly["wv"] @ xn).astype(np.float32)
            q = rope(q, self.nh_l, hd, hd, pos, self.theta)
            k = rope(k, self.nkv_l, hd, hd, pos, self.theta)
            # kv_turboquant_encode (layer_scheduler.c:101-118), global amax
            amax = allmax(np.array([np.abs(k).max(), np.abs(v).max()], np.float32))
            for vec, cache, sc, a in ((k, self.kc, self.ks, amax[0]), (v, self.vc, self.vs, amax[1])):
                scale = np.float32(a / np.float32(127.0))
                inv = np.float32(1.0) / scale if scale > 0 else np.float32(0.0)
                cache[l, pos] = np.clip(np.floor(np.abs(vec * inv) + 0.5) * np.sign(vec * inv), -128, 127)
                sc[l, pos] = scale
            att = np.zeros(self.nh_l * hd, np.float32)
            for hq in range(self.nh_l):
                kvh = hq // G
                K = self.kc[l, :pos + 1, kvh * hd:(kvh + 1) * hd].astype(np.float32) * self.ks[l, :pos + 1, None]
                Vv = self.vc[l, :pos + 1, kvh * hd:(kvh + 1) * hd].astype(np.float32) * self.vs[l, :pos + 1, None]
                s = (K @ q[hq * hd:(hq + 1) * hd]).astype(np.float32) * np.float32(1.0 / np.sqrt(np.float32(hd)))
                e = np.exp(s - s.max()).astype(np.float32)
                p = e / e.sum(dtype=np.float32)
                att[hq * hd:(hq + 1) * hd] = (p @ Vv).astype(np.float32)
            part = (ly["wo"] @ att).astype(np.float32)
            h = allsum(part + h if self.rank == 0 else part)
            xn = rmsnorm(h, ly["fn"], self.eps)
            g = (ly["wg"] @ xn).astype(np.float32)
            u = (ly["wu"] @ xn).astype(np.float32)
            act = (u * (g / (np.float32(1.0) + np.exp(-g)))).astype(np.float32)
            part = (ly["wd"] @ act).astype(np.float32)
            h = allsum(part + h if self.rank == 0 else part)
        xn = rmsnorm(h, self.out_norm, self.eps)
        logits = (self.head @ xn).astype(np.float32)
        best = max(pack_argmax(float(x), self.rank * self.Vl + i) for i, x in enumerate(logits))
        best = allbest(best)
        return 0x7FFFFFFF - (best & 0xFFFFFFFF), logits


def model_dims(path: str, cfg) -> dict:
    return dict(d=cfg.d_model, L=cfg.n_layers, nh=cfg.n_heads, nkv=cfg.n_kv_heads, hd=cfg.head_dim,
                ff=cfg.ffn, V=cfg.vocab, eps=cfg.rms_eps, theta=cfg.rope_theta)


def run_local(path: str, cfg, tp: int, prompt, steps: int, ctx: int = 64):
    """All `tp` ranks in this process (rank-order sums, max over ranks);
    returns the greedy IDs (the first one after the prompt) and the full
    logits of every step (the ranks' slices concatenated)."""
    w = dequantized(path)
    dims = model_dims(path, cfg)
    shards = [Shard(w, dims, r, tp, ctx) for r in range(tp)]
    ids, all_logits = [], []
    pos = 0
    toks = list(prompt)
    for t in range(len(prompt) + steps - 1):
        tok = toks[t] if t < len(prompt) else ids[-1]
        outs = _step_all(shards, tok, pos)
        pos += 1
        if t >= len(prompt) - 1:
            ids.append(outs[0][0])
            all_logits.append(np.concatenate([o[1] for o in outs]))
    return ids, all_logits


def _step_all(shards, tok, pos):
    """Runs every rank's step in lockstep with generator-free exchanges: each
    exchange is computed from all ranks' contributions in rank order."""
    import threading
    n = len(shards)
    bar = threading.Barrier(n)
    slots = [None] * n
    results = [None] * n

    def exch(r, x, op):
        slots[r] = x
        bar.wait()
        vals = list(slots)
        bar.wait()
        if op == "max":
            return np.maximum.reduce(vals)
        if op == "sum":
            acc = vals[0].copy()
            for v in vals[1:]:
                acc = (acc + v).astype(np.float32)
            return acc
        return max(vals)

    def run(r):
        results[r] = shards[r].step(tok, pos, lambda x: exch(r, x, "max"), lambda x: exch(r, x, "sum"),
                                    lambda k: exch(r, k, "best"))

    th = [threading.Thread(target=run, args=(r,)) for r in range(n)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    return results
