"""CPU, world_size 2 and 3 over gloo: the vocab-sharded host protocol of
tabby_b200/sharded.py (slice bounds, rank-major all-gather of the per-shard blocks, the
merge every rank runs). The per-shard GPU step is stood in for by the oracle's block
(this container has no GPU); the GPU kernels behind the same protocol are checked in
tests/test_golden.py and tests/test_gpu_sharded.py."""
import os
import socket

import numpy as np
import pytest

from tabby_b200.sharded import BLOCK_WORDS, shard_bounds


def test_shard_bounds_partition_the_vocab():
    for V in (7, 1000, 49152, 151936):
        for P in (p for p in (1, 2, 3, 4, 8) if p <= V):
            spans = [shard_bounds(V, P, r) for r in range(P)]
            assert spans[0][0] == 0 and spans[-1][1] == V
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(3, 4, 0)
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle
        from tabby_b200 import synth
        from tabby_b200.sharded import gather_blocks

        x, p, u = synth.config("c5", seed=3, rows=4)
        lo, hi = shard_bounds(x.shape[1], world, rank)
        local = torch.from_numpy(oracle.shard_local_block(x[:, lo:hi], lo))
        assert local.shape == (4, BLOCK_WORDS)
        gathered = gather_blocks(local)
        out, ids, vals = oracle.shard_merge(gathered.numpy(), world, p, u)
        np.savez(f"{result_path}.{rank}.npz", out=out.view(np.uint8), ids=ids, vals=vals,
                 gathered=gathered.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_sharded_protocol_matches_whole_row(tmp_path, world):
    import torch.multiprocessing as mp

    from oracle import oracle
    from tabby_b200 import synth

    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, join=True,
                       start_method="spawn")
    res = [np.load(f"{path}.{r}.npz") for r in range(world)]
    for r in range(1, world):  # every rank ends with the same gathered blocks and tokens
        np.testing.assert_array_equal(res[r]["gathered"], res[0]["gathered"])
        np.testing.assert_array_equal(res[r]["out"], res[0]["out"])
    # Rank-major layout: block (shard s, row r) at s * rows + r, carrying global indices.
    x, p, u = synth.config("c5", seed=3, rows=4)
    g = res[0]["gathered"]
    for s in range(world):
        lo, hi = shard_bounds(x.shape[1], world, s)
        idx = g[s * 4:(s + 1) * 4, 3::2].view(np.uint32)
        assert ((idx >= lo) & (idx < hi)).all()
    out = res[0]["out"].view(oracle.OUTCOME_DTYPE)
    whole, wids, _ = oracle.sample_rows(x, p, u, 64)
    np.testing.assert_array_equal(out["id"], whole["id"])
    np.testing.assert_array_equal(out["considered_count"], whole["considered_count"])
    for r in range(4):
        n = int(whole[r]["pool_size"])
        np.testing.assert_array_equal(res[0]["ids"][r, :n], wids[r, :n])
    np.testing.assert_allclose(out["sum_exp"], whole["sum_exp"], rtol=1e-5)
    np.testing.assert_allclose(out["probability"], whole["probability"], rtol=1e-5)
