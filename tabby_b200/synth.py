"""Seeded synthetic logits and per-row parameters for the benchmark configurations.

The reference measures sampling on real model logits (Qwen2.5-0.5B, V=151936;
SmolLM2-360M, V=49152). No weights exist here, so seeded synthetic rows with those
shapes and the value distributions below stand in for them. Generator: numpy's PCG64
(seeded per config), normals by numpy's float32 standard_normal.

  c1  1 x 151936   fp32 N(0, 3^2)                          T 0.8, k 40, p 0.95
  c2  1 x 49152    N(0, 2^2) rounded to fp16 and widened; 8 random positions forced to
                   the row max (exact ties)               T 1.0, k in {1, 50}, p 1.0
  c3  64 x 151936  -1.1*ln(rank) + N(0, 0.5^2), ranks permuted per row
                                                           T 1.0, p 0.9, k in {1,8,64,256,1024}
  c4  256 x 151936 bf16(N(0, 4^2)) widened; 5% of rows get +12 on one random token
                   per row T ~ U[0.3, 1.5], k in {0, 20, 100, 1000}, p ~ U[0.5, 1.0]
  c5  512 x 151936 N(0, 3^2) + the c3 Zipf tail, split in contiguous vocab shards
                                                           T 0.7, k 50, p 0.9
Uniform draws: one per row from mulberry32 (SeededRandom) seeded with the config seed.
"""
from __future__ import annotations

import numpy as np

from ._lib import PARAMS_DTYPE
from .sampler import SeededRandom

VOCAB_QWEN = 151936
VOCAB_SMOL = 49152


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def round_fp16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).astype(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, widened back to float32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    b = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return b.view(np.float32)


def zipf_tail(g: np.random.Generator, rows: int, vocab: int) -> np.ndarray:
    """-1.1 * ln(rank) with ranks 1..V randomly permuted per row."""
    base = (-1.1 * np.log(np.arange(1, vocab + 1, dtype=np.float64))).astype(np.float32)
    out = np.empty((rows, vocab), np.float32)
    for r in range(rows):
        out[r] = base[g.permutation(vocab)]
    return out


def uniforms(seed: int, rows: int) -> np.ndarray:
    rng = SeededRandom(seed)
    return np.array([rng.next() for _ in range(rows)], np.float64)


def params(rows: int, temperature, top_p, top_k) -> np.ndarray:
    p = np.zeros(rows, PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_p"] = top_p
    p["top_k"] = top_k
    return p


def config(name: str, seed: int = 0, rows: int | None = None, vocab: int | None = None,
           top_k: int | None = None):
    """(logits float32 [rows, vocab], params PARAMS_DTYPE [rows], uniforms f64 [rows])."""
    g = _rng(seed * 1000 + int(name[1:]))
    if name == "c1":
        rows, vocab = rows or 1, vocab or VOCAB_QWEN
        x = (3.0 * g.standard_normal((rows, vocab), dtype=np.float32)).astype(np.float32)
        p = params(rows, 0.8, 0.95, 40 if top_k is None else top_k)
    elif name == "c2":
        rows, vocab = rows or 1, vocab or VOCAB_SMOL
        x = round_fp16(2.0 * g.standard_normal((rows, vocab), dtype=np.float32))
        for r in range(rows):
            pos = g.choice(vocab, 8, replace=False)
            x[r, pos] = x[r].max()
        p = params(rows, 1.0, 1.0, 50 if top_k is None else top_k)
    elif name == "c3":
        rows, vocab = rows or 64, vocab or VOCAB_QWEN
        x = zipf_tail(g, rows, vocab) + (0.5 * g.standard_normal((rows, vocab), dtype=np.float32)).astype(np.float32)
        p = params(rows, 1.0, 0.9, 64 if top_k is None else top_k)
    elif name == "c4":
        rows, vocab = rows or 256, vocab or VOCAB_QWEN
        x = round_bf16(4.0 * g.standard_normal((rows, vocab), dtype=np.float32))
        spike = g.random(rows) < 0.05
        for r in np.nonzero(spike)[0]:
            x[r, g.integers(vocab)] += 12.0
        p = np.zeros(rows, PARAMS_DTYPE)
        p["temperature"] = g.uniform(0.3, 1.5, rows)
        p["top_k"] = g.choice(np.array([0, 20, 100, 1000]), rows) if top_k is None else top_k
        p["top_p"] = g.uniform(0.5, 1.0, rows)
    elif name == "c5":
        rows, vocab = rows or 512, vocab or VOCAB_QWEN
        x = (3.0 * g.standard_normal((rows, vocab), dtype=np.float32)).astype(np.float32) + zipf_tail(g, rows, vocab)
        p = params(rows, 0.7, 0.9, 50 if top_k is None else top_k)
    else:
        raise ValueError(f"unknown config {name!r}")
    return np.ascontiguousarray(x, np.float32), p, uniforms(seed + 7, rows)
