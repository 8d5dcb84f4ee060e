"""Vocab-sharded sampling across GPUs (one process per GPU, torch.distributed over NCCL).

The reference samples a single row on one device (forward.ts:520-601); when an LM head
is split by tensor parallelism each rank holds a contiguous slice of every row's
logits. The exchange is one collective:

1. every rank runs tabby_shard_local_async on its slice -> per row a block
   [local max, local sum(exp(x - local max)), (value, global index) x 64];
2. one all-gather of those blocks (rank-major, (2 + 2*64) * 4 bytes per row per rank);
3. every rank runs tabby_shard_merge_async on the gathered blocks: M = max m_s,
   S = sum s_s * exp(m_s - M), the global top-k of the 64*P candidates by
   (value desc, global index asc), then sampleFromTopK (sampler.ts:147-212).

The (max, sum-exp) pairs travel inside the gathered blocks, so no separate all-reduce
is needed; every rank computes the same merge and ends with the same token ids (the
merge is deterministic), so no broadcast is needed either. Pool sizes are capped at
64 (TABBY_SHARD_TOP_K), the reference's MAX_TOP_K (kernels.ts:448).

With ``exchange="peer"`` steps 2 and 3 are one kernel instead: each rank's blocks stay in
its own CUDA-IPC-shared buffer (two, used in turn), and tabby_exchange_merge_async
announces them with a release store into every peer's flag word, waits for the peers'
words and merges every row reading the peers' blocks over NVLink, so no collective
library call is on the path.

Row-split data parallelism (independent rows per GPU) needs nothing from this module:
each rank runs Sampler.sample_batch on its own rows with no collective.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple, Union

import numpy as np

from . import _lib
from ._lib import OUTCOME_DTYPE, check, lib
from .sampler import SampleBatch, Sampler, SamplingParams, _raise_row_errors, params_array

SHARD_TOP_K = 64  # TABBY_SHARD_TOP_K in include/tabby_sample.h
BLOCK_WORDS = 2 + 2 * SHARD_TOP_K


def shard_bounds(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, nearly equal slices: rank r owns [r*V//P, (r+1)*V//P)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if vocab < world:
        raise ValueError(f"vocab {vocab} smaller than world size {world}")
    return rank * vocab // world, (rank + 1) * vocab // world


def gather_blocks(block, group=None):
    """All-gather per-rank [rows, W] float32 blocks into [world * rows, W], rank-major
    (the layout tabby_shard_merge_async reads). NCCL gathers into one flat buffer;
    other backends (gloo on CPU) gather a list and concatenate."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows, width = block.shape
    block = block.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * rows, width), dtype=block.dtype, device=block.device)
        dist.all_gather_into_tensor(out, block, group=group)
        return out
    parts = [torch.empty_like(block) for _ in range(world)]
    dist.all_gather(parts, block, group=group)
    return torch.cat(parts, 0)


class PeerExchange:
    """This rank's tabby_exchange: a CUDA-IPC-shared buffer that every rank of `group`
    maps, for tabby_exchange_merge_async. Collective to construct (every rank at once)."""

    def __init__(self, device: int, max_rows: int, group=None):
        import ctypes

        import torch.distributed as dist

        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.group = group
        h = ctypes.c_void_p()
        check(lib().tabby_exchange_create(int(device), self.world, self.rank, int(max_rows),
                                          ctypes.byref(h)))
        self.handle = h
        self.max_rows = int(max_rows)
        try:
            mine = ctypes.create_string_buffer(_lib.TABBY_EXCHANGE_HANDLE_BYTES)
            check(lib().tabby_exchange_ipc_handle(h, mine))
            if self.world > 1:
                allh = [None] * self.world
                dist.all_gather_object(allh, mine.raw, group=group)
            else:
                allh = [mine.raw]
            blob = ctypes.create_string_buffer(b"".join(allh), len(allh) * len(mine.raw))
            check(lib().tabby_exchange_open(h, blob))
        except Exception:
            lib().tabby_exchange_destroy(h)
            raise

    def next_blocks(self):
        """(device pointer, row stride in words) of the block buffer the next merge reads
        (the two buffers alternate from step to step)."""
        import ctypes

        ptr, ld = ctypes.c_void_p(), ctypes.c_int32()
        check(lib().tabby_exchange_blocks(self.handle, ctypes.byref(ptr), ctypes.byref(ld)))
        return ptr.value, ld.value

    def close(self) -> None:
        """Frees the buffer; call on every rank after a barrier that follows the last merge."""
        if self.handle:
            lib().tabby_exchange_destroy(self.handle)
            self.handle = None


class ShardedSampler:
    """Sampling of vocab-sharded rows on this rank's GPU; one instance per rank.

    exchange: "gather" (NCCL all-gather of the blocks, then every rank merges every row)
    or "peer" (PeerExchange: the merge kernel reads the peers' blocks over peer memory
    itself after one flag handshake)."""

    def __init__(self, vocab: int, device: Optional[int] = None, group=None,
                 max_rows: int = 512, exchange: str = "gather"):
        import torch
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.vocab = int(vocab)
        self.lo, self.hi = shard_bounds(self.vocab, self.world, self.rank)
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.sampler = Sampler(self.device, max_top_k=SHARD_TOP_K, max_rows=max_rows,
                               max_vocab=self.hi - self.lo)
        if exchange not in ("gather", "peer"):
            raise ValueError(f"exchange must be 'gather' or 'peer', got {exchange!r}")
        self.exchange = PeerExchange(self.device, max_rows, group) if exchange == "peer" else None

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
        self.sampler.close()

    def local_into_exchange(self, local_logits) -> int:
        """Step 1 into the peer exchange buffer; returns the row count."""
        x = self.sampler._check_logits(local_logits)
        rows, sv = x.shape
        if sv != self.hi - self.lo:
            raise ValueError(f"rank {self.rank} holds {self.hi - self.lo} columns, got {sv}")
        if rows > self.exchange.max_rows:
            raise ValueError(f"{rows} rows exceed the exchange's {self.exchange.max_rows}")
        blocks, ld = self.exchange.next_blocks()
        check(lib().tabby_shard_local_async(self.sampler.handle, x.data_ptr(), x.stride(0), rows,
                                            sv, self.lo, blocks, ld, self.sampler._stream()))
        return rows

    def exchange_merge_async(self, rows: int, params_dev, uniforms_dev, out_dev) -> None:
        """Steps 2-3 in one kernel over peer memory (device tensors, no sync); every rank
        must call it once per local_into_exchange, in the same order."""
        check(lib().tabby_exchange_merge_async(self.exchange.handle, rows, params_dev.data_ptr(),
                                               uniforms_dev.data_ptr(), out_dev.data_ptr(),
                                               self.sampler._stream()))

    def local_blocks(self, local_logits):
        """Step 1: [rows, 130] float32 blocks of this rank's slice (device tensor)."""
        import torch

        x = self.sampler._check_logits(local_logits)
        rows, sv = x.shape
        if sv != self.hi - self.lo:
            raise ValueError(f"rank {self.rank} holds {self.hi - self.lo} columns, got {sv}")
        block = torch.empty((rows, BLOCK_WORDS), dtype=torch.float32, device=x.device)
        check(lib().tabby_shard_local_async(self.sampler.handle, x.data_ptr(), x.stride(0), rows,
                                            sv, self.lo, block.data_ptr(), BLOCK_WORDS,
                                            self.sampler._stream()))
        return block

    def merge_async(self, gathered, shards: int, params_dev, uniforms_dev, out_dev,
                    topk_ids=None, topk_values=None) -> None:
        """Step 3 on device tensors (no sync)."""
        rows = gathered.shape[0] // shards
        ld = topk_ids.shape[1] if topk_ids is not None else (
            topk_values.shape[1] if topk_values is not None else 0)
        check(lib().tabby_shard_merge_async(
            self.sampler.handle, gathered.data_ptr(), shards, rows, gathered.stride(0),
            params_dev.data_ptr(), uniforms_dev.data_ptr(), out_dev.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_values.data_ptr() if topk_values is not None else None, ld,
            self.sampler._stream()))

    def sample_batch(self, local_logits,
                     params: Union[SamplingParams, Sequence[SamplingParams]],
                     uniforms: np.ndarray, return_topk: bool = False) -> SampleBatch:
        """One token per row from this rank's slice; identical result on every rank."""
        import torch

        if self.exchange is not None:
            if return_topk:
                raise ValueError("return_topk needs exchange='gather'")
            rows = self.local_into_exchange(local_logits)
            dev = torch.device("cuda", self.device)
        else:
            block = self.local_blocks(local_logits)
            rows = block.shape[0]
            gathered = gather_blocks(block, self.group)
            dev = block.device
        p = params_array(params, rows)
        u = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(-1)
        if u.size != rows:
            raise ValueError(f"{u.size} uniforms for {rows} rows")
        p_dev = torch.from_numpy(p.view(np.uint8)).to(dev)
        u_dev = torch.from_numpy(u).to(dev)
        out_dev = torch.empty(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        if self.exchange is not None:
            self.exchange_merge_async(rows, p_dev, u_dev, out_dev)
            out = out_dev.cpu().numpy().view(OUTCOME_DTYPE)
            _raise_row_errors(out)
            return SampleBatch(out["id"].copy(), out, None, None)
        ids_dev = vals_dev = None
        if return_topk:
            ids_dev = torch.full((rows, SHARD_TOP_K), -1, dtype=torch.int32, device=dev)
            vals_dev = torch.zeros((rows, SHARD_TOP_K), dtype=torch.float32, device=dev)
        self.merge_async(gathered, self.world, p_dev, u_dev, out_dev, ids_dev, vals_dev)
        out = out_dev.cpu().numpy().view(OUTCOME_DTYPE)
        _raise_row_errors(out)
        return SampleBatch(out["id"].copy(), out,
                           ids_dev.cpu().numpy() if return_topk else None,
                           vals_dev.cpu().numpy() if return_topk else None)


__all__ = ["SHARD_TOP_K", "BLOCK_WORDS", "shard_bounds", "gather_blocks", "PeerExchange",
           "ShardedSampler"]
_ = _lib  # status constants live there
