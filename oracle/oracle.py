"""TEST INFRASTRUCTURE ONLY: ctypes wrapper around the C parity oracle (liboracle.so).

The oracle restates the reference's CPU sampler (xOAviOx/tabby src/engine/sampler.ts
:13-30, :105-119, :147-212 and src/worker/inference.worker.ts:120-123). Only tests/,
``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg import this module; the
product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

PARAMS_DTYPE = np.dtype(
    [("temperature", "<f8"), ("top_p", "<f8"), ("top_k", "<i4"), ("reserved", "<i4")]
)
OUTCOME_DTYPE = np.dtype(
    [
        ("id", "<i4"),
        ("considered_count", "<i4"),
        ("probability", "<f8"),
        ("pool_mass", "<f8"),
        ("pool_exhausted", "<i4"),
        ("pool_size", "<i4"),
        ("max_logit", "<f4"),
        ("sum_exp", "<f4"),
        ("status", "<i4"),
        ("reserved", "<i4"),
    ]
)

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc only; no GPU)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "sampler_ref.c")
        if not os.path.exists(_LIB_PATH) or (
            os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)
        ):
            build()
        l = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        l.or_mulberry32_u32.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        l.or_mulberry32_u32.restype = ctypes.c_uint32
        l.or_mulberry32_next.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        l.or_mulberry32_next.restype = ctypes.c_double
        l.or_js_exp.argtypes = [ctypes.c_double]
        l.or_js_exp.restype = ctypes.c_double
        l.or_argmax.argtypes = [P, ctypes.c_int64]
        l.or_argmax.restype = ctypes.c_int32
        l.or_topk.argtypes = [P, ctypes.c_int64, ctypes.c_int32, P, P]
        l.or_topk.restype = ctypes.c_int32
        l.or_pool_size.argtypes = [ctypes.c_double, ctypes.c_int32, ctypes.c_int32]
        l.or_pool_size.restype = ctypes.c_int32
        l.or_row_max.argtypes = [P, ctypes.c_int64]
        l.or_row_max.restype = ctypes.c_float
        l.or_sum_exp_f64.argtypes = [P, ctypes.c_int64, ctypes.c_float]
        l.or_sum_exp_f64.restype = ctypes.c_double
        l.or_sum_exp_wgsl_f32.argtypes = [P, ctypes.c_int64, ctypes.c_float]
        l.or_sum_exp_wgsl_f32.restype = ctypes.c_float
        l.or_sample_from_topk.argtypes = [
            P, P, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
            ctypes.c_double, ctypes.c_double, ctypes.c_double, P,
        ]
        l.or_sample_from_topk.restype = ctypes.c_int
        l.or_sample_rows.argtypes = [
            P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, P, P, ctypes.c_int32,
            P, P, P, ctypes.c_int32, ctypes.c_int32,
        ]
        l.or_sample_rows.restype = ctypes.c_int
        l.or_bench_rows.argtypes = [
            P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, P, P, ctypes.c_int32,
            ctypes.c_int32,
        ]
        l.or_bench_rows.restype = ctypes.c_double
        _lib = l
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class SeededRandom:
    """mulberry32, as sampler.ts:105-119."""

    def __init__(self, seed: int):
        self._state = ctypes.c_uint32(seed & 0xFFFFFFFF)

    def next(self) -> float:
        return lib().or_mulberry32_next(ctypes.byref(self._state))

    def next_u32(self) -> int:
        return lib().or_mulberry32_u32(ctypes.byref(self._state))


def js_exp(x: float) -> float:
    return lib().or_js_exp(float(x))


def argmax(row: np.ndarray) -> int:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return lib().or_argmax(_ptr(row), row.size)


def topk(row: np.ndarray, k: int):
    row = np.ascontiguousarray(row, dtype=np.float32)
    ids = np.zeros(max(k, 1), np.int32)
    vals = np.zeros(max(k, 1), np.float32)
    n = lib().or_topk(_ptr(row), row.size, k, _ptr(ids), _ptr(vals))
    return ids[:n], vals[:n]


def pool_size(temperature: float, top_k: int, cap: int) -> int:
    return lib().or_pool_size(float(temperature), int(top_k), int(cap))


def row_max(row: np.ndarray) -> float:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return lib().or_row_max(_ptr(row), row.size)


def sum_exp_f64(row: np.ndarray, mx: float) -> float:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return lib().or_sum_exp_f64(_ptr(row), row.size, mx)


def sum_exp_wgsl_f32(row: np.ndarray, mx: float) -> float:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return lib().or_sum_exp_wgsl_f32(_ptr(row), row.size, mx)


def sample_from_topk(ids, logits, max_logit, sum_exp, temperature, top_p, u) -> dict:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.zeros(1, OUTCOME_DTYPE)
    rc = lib().or_sample_from_topk(
        _ptr(ids), _ptr(logits), ids.size, float(max_logit), float(sum_exp),
        float(temperature), float(top_p), float(u), _ptr(out),
    )
    if rc != 0:
        raise ValueError("sampleFromTopK: empty candidate set")
    o = out[0]
    return {
        "id": int(o["id"]),
        "probability": float(o["probability"]),
        "consideredCount": int(o["considered_count"]),
        "poolMass": float(o["pool_mass"]),
        "poolExhausted": bool(o["pool_exhausted"]),
    }


def make_params(temperature, top_p, top_k, rows: int) -> np.ndarray:
    p = np.zeros(rows, PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_p"] = top_p
    p["top_k"] = top_k
    return p


def sample_rows(logits: np.ndarray, params: np.ndarray, uniforms: np.ndarray, cap: int,
                threads: int = os.cpu_count() or 1):
    """Reference path for every row: returns (outcomes, topk_ids, topk_values)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float64)
    out = np.zeros(rows, OUTCOME_DTYPE)
    ids = np.full((rows, cap), -1, np.int32)
    vals = np.zeros((rows, cap), np.float32)
    rc = lib().or_sample_rows(
        _ptr(logits), vocab, rows, vocab, _ptr(params), _ptr(uniforms), cap,
        _ptr(out), _ptr(ids), _ptr(vals), cap, threads,
    )
    if rc != 0:
        raise ValueError("or_sample_rows: invalid arguments")
    return out, ids, vals


def bench_rows(logits: np.ndarray, params: np.ndarray, uniforms: np.ndarray, cap: int,
               threads: int) -> float:
    """Seconds the reference CPU path takes over all rows of ``logits``."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float64)
    return lib().or_bench_rows(
        _ptr(logits), vocab, rows, vocab, _ptr(params), _ptr(uniforms), cap, threads
    )


# ---------------------------------------------------------------------------------------
# Vocab-sharded sampling (a multi-GPU protocol new in this build; the reference samples
# one row on one device). The restatement below defines what the sharded path must equal:
# local (max, sum-exp, top-64) per shard, then M = max m_s, S = sum s_s * exp(m_s - M),
# the global top-k by (value desc, index asc) and sampleFromTopK (sampler.ts:147-212).
# ---------------------------------------------------------------------------------------
SHARD_TOP_K = 64


def shard_local_block(x: np.ndarray, offset: int) -> np.ndarray:
    """[rows, 2 + 2*64] float32 blocks for the columns [offset, offset + x.shape[1])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    blk = np.zeros((rows, 2 + 2 * SHARD_TOP_K), np.float32)
    u = blk.view(np.uint32)
    for r in range(rows):
        m = row_max(x[r])
        blk[r, 0] = m
        blk[r, 1] = np.float32(sum_exp_f64(x[r], m))
        ids, vals = topk(x[r], SHARD_TOP_K)
        blk[r, 2::2] = -np.inf
        u[r, 3::2] = 0xFFFFFFFF
        blk[r, 2:2 + 2 * ids.size:2] = vals
        u[r, 3:3 + 2 * ids.size:2] = (ids.astype(np.int64) + offset).astype(np.uint32)
    return blk


def shard_merge(blocks: np.ndarray, shards: int, params: np.ndarray, uniforms: np.ndarray):
    """blocks: [shards * rows, 130] rank-major. Returns (outcomes, topk_ids, topk_values)."""
    import math

    blocks = np.ascontiguousarray(blocks, dtype=np.float32)
    rows = blocks.shape[0] // shards
    u32 = blocks.view(np.uint32)
    out = np.zeros(rows, OUTCOME_DTYPE)
    tids = np.full((rows, SHARD_TOP_K), -1, np.int32)
    tvals = np.zeros((rows, SHARD_TOP_K), np.float32)
    for r in range(rows):
        b = [blocks[s * rows + r] for s in range(shards)]
        bu = [u32[s * rows + r] for s in range(shards)]
        M = max(float(x[0]) for x in b)
        S = 0.0
        for x in b:
            if x[1] > 0:
                S += float(x[1]) * js_exp(float(x[0]) - M)
        cand = []
        for x, xu in zip(b, bu):
            for j in range(SHARD_TOP_K):
                if xu[3 + 2 * j] != 0xFFFFFFFF:
                    v = float(x[2 + 2 * j])
                    cand.append((-(v + 0.0), int(xu[3 + 2 * j]), x[2 + 2 * j]))
        cand.sort(key=lambda c: (c[0], c[1]))
        p = params[r]
        k = min(pool_size(p["temperature"], p["top_k"], SHARD_TOP_K), len(cand))
        ids = np.array([c[1] for c in cand[:k]], np.int32)
        vals = np.array([c[2] for c in cand[:k]], np.float32)
        o = np.zeros(1, OUTCOME_DTYPE)
        rc = lib().or_sample_from_topk(
            _ptr(ids), _ptr(vals), k, float(vals[0]) if k else M, float(np.float32(S)),
            float(p["temperature"]), float(p["top_p"]), float(uniforms[r]), _ptr(o))
        if rc != 0:
            raise ValueError("sampleFromTopK: empty candidate set")
        o["pool_size"] = k
        out[r] = o[0]
        tids[r, :k] = ids
        tvals[r, :k] = vals
    return out, tids, tvals


def softmax_rows(x: np.ndarray, n_rows: int, row_len: int, causal_period: int = 0,
                 causal_offset: int = 0) -> np.ndarray:
    """Restatement of cpu.ts:238-264 (softmaxRows, the CPU form of softmax_rows.wgsl) with
    its fp32 rounding (f32 = Math.fround, cpu.ts:17): per row, max over the kept prefix,
    e = f32(exp(f32(x - max))) with the exp in float64, sum = f32(sum + e) left to right,
    inv = f32(1 / sum), out = f32(e * inv); entries past the prefix become 0."""
    src = np.ascontiguousarray(x, np.float32).reshape(n_rows, row_len)
    out = src.copy()
    for r in range(n_rows):
        valid = causal_offset + (r % causal_period) + 1 if causal_period else row_len
        row = src[r, :valid]
        mx = np.float32(row.max())
        e = np.exp((row - mx).astype(np.float32).astype(np.float64)).astype(np.float32)
        s = np.float32(0.0)
        for v in e:  # left to right, every step rounded to fp32
            s = np.float32(s + v)
        inv = np.float32(np.float64(1.0) / np.float64(s))
        out[r, :valid] = (e * inv).astype(np.float32)
        out[r, valid:] = 0.0
    return out
