"""Host-side mirror of the reference sampler API over the CUDA library.

Mirrors xOAviOx/tabby src/engine/sampler.ts: ``SamplingParams`` (:83-91),
``DEFAULT_SAMPLING`` (:93-98), ``SeededRandom`` (:105-119), ``SampleOutcome`` (:121-135),
``sampleFromTopK`` (:147-212), and the GPU half ``TopKResult`` (src/engine/forward.ts
:94-103) produced by ``ForwardPass.runFull(ids, {topK})``. ``Sampler.sample(logits,
params, rng)`` is the drop-in call: the GPU computes max, sum-exp, the exact top-k and the
float64 sampleFromTopK in one launch and returns the token id.

Device memory, streams and the process group come from PyTorch; the compute is the C-ABI
library (``tabby_b200/lib/libtabbysample.so``). There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Union

import numpy as np

from . import _lib
from ._lib import OUTCOME_DTYPE, PARAMS_DTYPE, TabbyError, check, lib

MAX_TOP_K = _lib.TABBY_DEFAULT_MAX_TOP_K  # src/engine/kernels.ts:448


@dataclass
class SamplingParams:
    """sampler.ts:83-91. ``topK`` 0 asks for the largest pool (MAX_TOP_K)."""

    temperature: float
    topK: int
    topP: float
    seed: int = 0


DEFAULT_SAMPLING = SamplingParams(temperature=0.7, topK=40, topP=0.9, seed=0)


class SeededRandom:
    """mulberry32 (sampler.ts:105-119); advanced once per sampled row."""

    def __init__(self, seed: int):
        self._state = seed & 0xFFFFFFFF

    def next_u32(self) -> int:
        self._state = (self._state + 0x6D2B79F5) & 0xFFFFFFFF
        t = self._state
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + (((t ^ (t >> 7)) * (t | 61)) & 0xFFFFFFFF)) & 0xFFFFFFFF
        return (t ^ (t >> 14)) & 0xFFFFFFFF

    def next(self) -> float:
        return self.next_u32() / 4294967296.0


@dataclass
class SampleOutcome:
    """sampler.ts:121-135."""

    id: int
    probability: float
    consideredCount: int
    poolMass: float
    poolExhausted: bool


@dataclass
class TopKResult:
    """forward.ts:94-103: candidates highest logit first, ties by lower id."""

    maxLogit: float
    sumExp: float
    ids: List[int] = field(default_factory=list)
    logits: List[float] = field(default_factory=list)


@dataclass
class SampleBatch:
    ids: np.ndarray                 # int32 [rows], the sampled tokens
    outcomes: np.ndarray            # OUTCOME_DTYPE [rows]
    topk_ids: Optional[np.ndarray] = None     # int32 [rows, max_top_k] (pool_size valid)
    topk_values: Optional[np.ndarray] = None  # float32 [rows, max_top_k]

    def outcome(self, r: int) -> SampleOutcome:
        o = self.outcomes[r]
        return SampleOutcome(int(o["id"]), float(o["probability"]), int(o["considered_count"]),
                             float(o["pool_mass"]), bool(o["pool_exhausted"]))


def pool_size(temperature: float, top_k: int, max_top_k: int = MAX_TOP_K) -> int:
    """Worker pool rule (src/worker/inference.worker.ts:120-123)."""
    return int(lib().tabby_pool_size(float(temperature), int(top_k), int(max_top_k)))


def params_array(params: Union[SamplingParams, Sequence[SamplingParams]], rows: int) -> np.ndarray:
    """Per-row tabby_sampling_params from one SamplingParams or one per row."""
    out = np.zeros(rows, PARAMS_DTYPE)
    if isinstance(params, SamplingParams):
        params = [params] * rows
    if len(params) != rows:
        raise ValueError(f"{len(params)} SamplingParams for {rows} rows")
    for r, p in enumerate(params):
        out[r] = (float(p.temperature), float(p.topP), int(p.topK), 0)
    return out


def sample_from_topk(top: TopKResult, params: SamplingParams,
                     random: SeededRandom) -> SampleOutcome:
    """sampleFromTopK (sampler.ts:147-212), same float64 arithmetic as the GPU finalize."""
    n = len(top.ids)
    if n == 0:
        raise ValueError("sampleFromTopK: empty candidate set")
    ids = np.ascontiguousarray(top.ids, dtype=np.int32)
    vals = np.ascontiguousarray(top.logits, dtype=np.float32)
    p = params_array(params, 1)
    out = np.zeros(1, OUTCOME_DTYPE)
    # The reference draws only when it samples: a greedy call returns before
    # random.next() (sampler.ts:159-167, the draw at :194), leaving the generator as it was.
    u = random.next() if float(params.temperature) > 0 else 0.0
    check(lib().tabby_sample_from_topk(ids.ctypes.data, vals.ctypes.data, n,
                                       float(top.maxLogit), float(top.sumExp), p.ctypes.data,
                                       u, out.ctypes.data))
    o = out[0]
    return SampleOutcome(int(o["id"]), float(o["probability"]), int(o["considered_count"]),
                         float(o["pool_mass"]), bool(o["pool_exhausted"]))


sampleFromTopK = sample_from_topk


def _torch():
    import torch  # plumbing only: device memory and streams

    return torch


class Sampler:
    """A sampler bound to one CUDA device (the GPU half of ForwardPass's sampling).

    ``max_top_k`` is the pool cap (MAX_TOP_K): 64 in the reference, up to 1024 here.
    ``max_rows``/``max_vocab`` size the staging of the host-buffer path.
    """

    def __init__(self, device: int = 0, max_top_k: int = MAX_TOP_K, max_rows: int = 256,
                 max_vocab: int = 151936):
        self.device = int(device)
        self.max_top_k = int(max_top_k)
        cfg = _lib.SamplerConfig(self.device, self.max_top_k, int(max_rows), int(max_vocab))
        handle = ctypes.c_void_p()
        check(lib().tabby_sampler_create(ctypes.byref(cfg), ctypes.byref(handle)))
        self._h = handle

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().tabby_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    # -- helpers --------------------------------------------------------------------
    def _stream(self) -> int:
        torch = _torch()
        return torch.cuda.current_stream(self.device).cuda_stream

    def _check_logits(self, logits):
        torch = _torch()
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.dim() != 2:
            raise ValueError("logits must be [vocab] or [rows, vocab]")
        if logits.dtype != torch.float32:
            raise TypeError("logits must be float32 (the lm_head output of forward.ts:416-426)")
        if not logits.is_cuda or logits.device.index != self.device:
            raise ValueError(f"logits must live on cuda:{self.device}")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        return logits

    @staticmethod
    def _uniforms(rows: int, rng: Union[SeededRandom, Sequence[float], np.ndarray, None],
                  p: Optional[np.ndarray] = None):
        """Per-row u. With a SeededRandom, rows are drawn in row order and only where
        sampleFromTopK itself would call random.next(): rows with temperature > 0. Greedy
        rows return before the draw in the reference (sampler.ts:159-167) and get u = 0
        without advancing the generator, exactly as the device-RNG entry point does."""
        if isinstance(rng, SeededRandom):
            temps = p["temperature"] if p is not None else np.ones(rows)
            return np.array([rng.next() if float(t) > 0 else 0.0 for t in temps[:rows]],
                            np.float64)
        if rng is None:
            raise ValueError("a SeededRandom or per-row uniforms are required")
        u = np.ascontiguousarray(rng, dtype=np.float64).reshape(-1)
        if u.size != rows:
            raise ValueError(f"{u.size} uniforms for {rows} rows")
        return u

    # -- device path ----------------------------------------------------------------
    def sample_rows_async(self, logits, params_dev, uniforms_dev, out_dev, topk_ids=None,
                          topk_values=None, stream: Optional[int] = None) -> None:
        """All-device call of tabby_sample_rows_async on torch tensors (no sync)."""
        logits = self._check_logits(logits)
        rows, vocab = logits.shape
        ld = topk_ids.shape[1] if topk_ids is not None else (
            topk_values.shape[1] if topk_values is not None else 0)
        check(lib().tabby_sample_rows_async(
            self._h, logits.data_ptr(), logits.stride(0), rows, vocab, params_dev.data_ptr(),
            uniforms_dev.data_ptr(), out_dev.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_values.data_ptr() if topk_values is not None else None, ld,
            self._stream() if stream is None else stream))

    def sample_rows_rng_async(self, logits, params_dev, rng_state_dev, out_dev, topk_ids=None,
                              topk_values=None, stream: Optional[int] = None) -> None:
        """tabby_sample_rows_rng_async on torch tensors (no sync): u drawn on the device
        from ``rng_state_dev`` (uint32 mulberry32 state per row, advanced in place exactly
        where SeededRandom.next() would be called). Graph-capturable."""
        logits = self._check_logits(logits)
        rows, vocab = logits.shape
        ld = topk_ids.shape[1] if topk_ids is not None else (
            topk_values.shape[1] if topk_values is not None else 0)
        check(lib().tabby_sample_rows_rng_async(
            self._h, logits.data_ptr(), logits.stride(0), rows, vocab, params_dev.data_ptr(),
            rng_state_dev.data_ptr(), out_dev.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_values.data_ptr() if topk_values is not None else None, ld,
            self._stream() if stream is None else stream))

    def sample_batch(self, logits, params: Union[SamplingParams, Sequence[SamplingParams]],
                     rng, return_topk: bool = False) -> SampleBatch:
        """Sample one token per row. ``logits`` is a CUDA tensor [rows, vocab] (device
        path) or a host numpy array (host-buffer path, copies inside)."""
        if isinstance(logits, np.ndarray):
            return self._sample_host(logits, params, rng, return_topk)
        torch = _torch()
        logits = self._check_logits(logits)
        rows = logits.shape[0]
        p = params_array(params, rows)
        u = self._uniforms(rows, rng, p)
        dev = logits.device
        p_dev = torch.from_numpy(p.view(np.uint8)).to(dev, non_blocking=False)
        u_dev = torch.from_numpy(u).to(dev)
        out_dev = torch.empty(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        ids_dev = vals_dev = None
        if return_topk:
            ids_dev = torch.full((rows, self.max_top_k), -1, dtype=torch.int32, device=dev)
            vals_dev = torch.zeros((rows, self.max_top_k), dtype=torch.float32, device=dev)
        self.sample_rows_async(logits, p_dev, u_dev, out_dev, ids_dev, vals_dev)
        out = out_dev.cpu().numpy().view(OUTCOME_DTYPE)
        _raise_row_errors(out)
        return SampleBatch(out["id"].copy(), out,
                           ids_dev.cpu().numpy() if return_topk else None,
                           vals_dev.cpu().numpy() if return_topk else None)

    def _sample_host(self, logits: np.ndarray, params, rng, return_topk: bool) -> SampleBatch:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        if logits.ndim == 1:
            logits = logits[None, :]
        rows, vocab = logits.shape
        p = params_array(params, rows)
        u = self._uniforms(rows, rng, p)
        out = np.zeros(rows, OUTCOME_DTYPE)
        ids = vals = None
        if return_topk:
            ids = np.full((rows, self.max_top_k), -1, np.int32)
            vals = np.zeros((rows, self.max_top_k), np.float32)
        check(lib().tabby_sample_rows(
            self._h, logits.ctypes.data, vocab, rows, vocab, p.ctypes.data, u.ctypes.data,
            out.ctypes.data, ids.ctypes.data if return_topk else None,
            vals.ctypes.data if return_topk else None, self.max_top_k if return_topk else 0))
        return SampleBatch(out["id"].copy(), out, ids, vals)

    def sample(self, logits, params: SamplingParams = DEFAULT_SAMPLING,
               rng: Optional[SeededRandom] = None) -> int:
        """The drop-in call: sample(logits, {temperature, topK, topP}, rng) -> token id."""
        if rng is None:
            rng = SeededRandom(params.seed)
        return int(self.sample_batch(logits, params, rng).ids[0])

    # -- TopKResult path (ForwardPass.runFull(ids, {topK})) ---------------------------
    def topk_block(self, logits, k: int):
        """[rows, 2 + 2k] float32 CUDA tensor: [maxLogit, sumExp, (value, idx bits) * k]."""
        torch = _torch()
        logits = self._check_logits(logits)
        rows, vocab = logits.shape
        block = torch.empty((rows, 2 + 2 * k), dtype=torch.float32, device=logits.device)
        check(lib().tabby_topk_rows_async(self._h, logits.data_ptr(), logits.stride(0), rows,
                                          vocab, int(k), block.data_ptr(), block.stride(0),
                                          self._stream()))
        return block

    def topk(self, logits, k: int) -> List[TopKResult]:
        """Decode the block like decodeSampleBlock (forward.ts:146-157)."""
        raw = self.topk_block(logits, k).cpu().numpy()
        return [decode_sample_block(raw[r], k) for r in range(raw.shape[0])]


def decode_sample_block(block: np.ndarray, k: int) -> TopKResult:
    """[maxLogit, sumExp, (value, index) * k]; the index is a u32 in an f32 slot."""
    f = np.ascontiguousarray(block, dtype=np.float32)
    u = f.view(np.uint32)
    return TopKResult(float(f[0]), float(f[1]), [int(u[3 + 2 * i]) for i in range(k)],
                      [float(f[2 + 2 * i]) for i in range(k)])


def _raise_row_errors(out: np.ndarray) -> None:
    bad = np.nonzero(out["status"] != _lib.TABBY_OK)[0]
    if bad.size:
        r = int(bad[0])
        st = int(out["status"][r])
        msg = {
            _lib.TABBY_EINPUT: "logits hold NaN, +-inf or a value <= -3.0e38",
            _lib.TABBY_EINVAL: "temperature or top_p is NaN",
            _lib.TABBY_ETIMEOUT: "a bounded device wait timed out",
            _lib.TABBY_EEMPTY: "sampleFromTopK: empty candidate set",
        }.get(st, "row failed")
        raise TabbyError(st, f"row {r}: {msg}")
