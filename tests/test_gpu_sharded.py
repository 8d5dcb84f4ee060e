"""GPU: vocab-sharded sampling through tabby_b200.sharded.ShardedSampler against the
oracle's whole-row result at pool cap 64: token ids, top-k sets and order bit-exact,
probabilities within 1e-5. Both exchanges are covered: the NCCL all-gather followed by
tabby_shard_merge_async ("gather"), and tabby_exchange_merge_async, whose kernel reads
the peers' blocks and writes the outcomes over peer memory ("peer").

Every world size runs as one process per GPU (spawned children, NVLS off) when the box
has that many GPUs (skipped otherwise). The peer exchange's bounded wait is also made to
run out: one rank never calls the merge, and the other's kernel must return with every
row reporting TABBY_ETIMEOUT."""
import os
import socket

import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu
REL = 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _compare(out, ids, x, p, u):
    from oracle import oracle

    whole, wids, wvals = oracle.sample_rows(x, p, u, 64)
    assert (out["status"] == 0).all()
    np.testing.assert_array_equal(out["id"], whole["id"])
    np.testing.assert_array_equal(out["considered_count"], whole["considered_count"])
    np.testing.assert_array_equal(out["pool_size"], whole["pool_size"])
    for r in range(x.shape[0]):
        n = int(whole[r]["pool_size"])
        np.testing.assert_array_equal(ids[r, :n], wids[r, :n])
    np.testing.assert_array_equal(out["max_logit"], whole["max_logit"])
    np.testing.assert_allclose(out["sum_exp"], whole["sum_exp"], rtol=REL)
    np.testing.assert_allclose(out["probability"], whole["probability"], rtol=REL)
    np.testing.assert_allclose(out["pool_mass"], whole["pool_mass"], rtol=REL)


def _rank_main(rank, world, port, rows, result_path, exchange="gather", calls=1):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        from tabby_b200 import synth
        from tabby_b200.sharded import ShardedSampler

        x, p, u = synth.config("c5", seed=11, rows=rows)
        s = ShardedSampler(x.shape[1], device=rank, max_rows=rows, exchange=exchange)
        local = torch.from_numpy(np.ascontiguousarray(x[:, s.lo:s.hi])).cuda(rank)
        from tabby_b200.sampler import SamplingParams

        params = [SamplingParams(float(q["temperature"]), int(q["top_k"]), float(q["top_p"]))
                  for q in p]
        outs = []
        for _ in range(calls):  # repeated calls reuse the buffers and flag words
            batch = s.sample_batch(local, params, u, return_topk=exchange == "gather")
            outs.append(batch.outcomes.view(np.uint8).copy())
        for o in outs[1:]:
            np.testing.assert_array_equal(o, outs[0])
        ids = batch.topk_ids if exchange == "gather" else np.zeros((0,), np.int32)
        np.savez(f"{result_path}.{rank}.npz", out=outs[0], ids=ids)
        torch.cuda.synchronize()
        dist.barrier()
        s.close()
    finally:
        dist.destroy_process_group()


def _run_world(tmp_path, world, rows, exchange="gather", calls=1):
    import torch

    if not gpu_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from oracle import oracle
    from tabby_b200 import synth

    path = str(tmp_path / "res")
    mp.start_processes(_rank_main, args=(world, _free_port(), rows, path, exchange, calls),
                       nprocs=world, join=True, start_method="spawn")
    res = [np.load(f"{path}.{r}.npz") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(res[r]["out"], res[0]["out"])
    x, p, u = synth.config("c5", seed=11, rows=rows)
    out = res[0]["out"].view(oracle.OUTCOME_DTYPE)
    if exchange == "gather":
        _compare(out, res[0]["ids"], x, p, u)
    else:
        whole, wids, _ = oracle.sample_rows(x, p, u, 64)
        _compare(out, wids, x, p, u)


def test_sharded_world1(tmp_path):
    _run_world(tmp_path, 1, 16)


def test_sharded_world2(tmp_path):
    _run_world(tmp_path, 2, 16)


def test_sharded_world4(tmp_path):
    _run_world(tmp_path, 4, 8)


def test_sharded_peer_world1(tmp_path):
    _run_world(tmp_path, 1, 16, "peer", calls=3)


def test_sharded_peer_world2(tmp_path):
    _run_world(tmp_path, 2, 37, "peer", calls=3)


def test_sharded_peer_world4(tmp_path):
    _run_world(tmp_path, 4, 9, "peer", calls=3)


def _timeout_main(rank, world, port, result_path):
    import time

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        from tabby_b200 import synth
        from tabby_b200._lib import OUTCOME_DTYPE
        from tabby_b200.sharded import ShardedSampler

        rows = 8
        x, p, u = synth.config("c5", seed=3, rows=rows)
        s = ShardedSampler(x.shape[1], device=rank, max_rows=rows, exchange="peer")
        local = torch.from_numpy(np.ascontiguousarray(x[:, s.lo:s.hi])).cuda(rank)
        s.local_into_exchange(local)
        dev = torch.device("cuda", rank)
        pd = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
        ud = torch.from_numpy(u).to(dev)
        out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        t0 = time.perf_counter()
        if rank == 0:  # rank 1 never joins the merge: rank 0's waits run out
            s.exchange_merge_async(rows, pd, ud, out)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        status = out.cpu().numpy().view(OUTCOME_DTYPE)["status"]
        np.savez(f"{result_path}.{rank}.npz", status=status, dt=np.array([dt]))
        dist.barrier()  # rank 1 keeps its buffer mapped until rank 0's kernel has returned
        s.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_wait_runs_out(tmp_path):
    import torch

    if not gpu_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from tabby_b200._lib import TABBY_ETIMEOUT

    path = str(tmp_path / "res")
    mp.start_processes(_timeout_main, args=(2, _free_port(), path), nprocs=2, join=True,
                       start_method="spawn")
    r0 = np.load(f"{path}.0.npz")
    assert (r0["status"] == TABBY_ETIMEOUT).all(), r0["status"]
    assert r0["dt"][0] < 5.0


def test_shard_merge_emulated_on_one_gpu():
    """8 shards of unequal, unaligned widths on one GPU, merged: equals the whole row."""
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import OUTCOME_DTYPE, check, lib
    from tabby_b200.sharded import BLOCK_WORDS, SHARD_TOP_K

    rows, P = 24, 8
    x, p, u = synth.config("c1", seed=5, rows=rows, vocab=100003)
    p["top_k"] = np.array([0, 1, 5, 50, 64, 100] * 4)
    p["temperature"] = np.array([0.0, 0.7, 1.0, 1.3] * 6)
    V = x.shape[1]
    cuts = [0, 1, 999, 12345, 40000, 40001, 77777, 99990, V]
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    blocks = torch.empty((P * rows, BLOCK_WORDS), dtype=torch.float32, device=dev)
    pd = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ids = torch.full((rows, SHARD_TOP_K), -1, dtype=torch.int32, device=dev)
    L = lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with Sampler(0, max_top_k=SHARD_TOP_K, max_rows=rows, max_vocab=V) as s:
        for sh in range(P):
            lo, hi = cuts[sh], cuts[sh + 1]
            check(L.tabby_shard_local_async(s.handle, xd[:, lo:].data_ptr(), V, rows, hi - lo,
                                            lo, blocks[sh * rows].data_ptr(), BLOCK_WORDS,
                                            stream))
        check(L.tabby_shard_merge_async(s.handle, blocks.data_ptr(), P, rows, BLOCK_WORDS,
                                        pd.data_ptr(), ud.data_ptr(), out.data_ptr(),
                                        ids.data_ptr(), None, SHARD_TOP_K, stream))
        torch.cuda.synchronize()
    _compare(out.cpu().numpy().view(OUTCOME_DTYPE), ids.cpu().numpy(), x, p, u)
