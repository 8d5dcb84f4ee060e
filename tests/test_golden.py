"""Golden fixtures (tests/golden/sampling_golden.json, made by make_golden.py there).

CPU: the oracle still reproduces every committed golden bit for bit, and the seeded
generator still yields the same logits (SHA-256). GPU: the product library, called
through the C ABI, matches every golden: token ids, top-k index sets and order and the
top-k values bit-exact; probabilities, pool mass and sum-exp within 1e-5 relative.
Sharded cases run all shards on one GPU (local blocks per slice, then the merge).
"""
import json
import os

import numpy as np
import pytest

from tests.conftest import gpu_available

HERE = os.path.dirname(os.path.abspath(__file__))
REL = 1e-5
GOLDEN = json.load(open(os.path.join(HERE, "golden", "sampling_golden.json")))
CASES = {c["name"]: c for c in GOLDEN["cases"]}


def _inputs(case):
    from tabby_b200 import synth

    return synth.config(case["config"], seed=case["seed"], rows=case["rows"],
                        top_k=case["top_k"])


def _check(case, out, ids, vals, exact_floats):
    for r, e in enumerate(case["expected"]):
        o = out[r]
        n = e["pool_size"]
        assert int(o["status"]) == 0
        assert int(o["id"]) == e["id"], (case["name"], r)
        assert int(o["considered_count"]) == e["considered_count"]
        assert int(o["pool_size"]) == n
        assert int(o["pool_exhausted"]) == e["pool_exhausted"]
        assert list(ids[r, :n]) == e["topk_ids"]
        assert np.ascontiguousarray(vals[r, :n]).view(np.uint32).tobytes().hex() == \
            e["topk_values_hex"]
        assert float(o["max_logit"]) == e["max_logit"]
        for key in ("probability", "pool_mass", "sum_exp"):
            if exact_floats:
                assert float(o[key]) == e[key], (case["name"], r, key)
            else:
                assert float(o[key]) == pytest.approx(e[key], rel=REL), (case["name"], r, key)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_reproduces_golden(oracle, name):
    import importlib.util

    case = CASES[name]
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    x, p, u = _inputs(case)
    assert mg.digest(x) == case["logits_sha256"], "synthetic generator changed"
    tup = next(c for c in mg.CASES if c[0] == name)
    out, ids, vals = mg.expected(tup, x, p, u)
    _check(case, out, ids, vals, exact_floats=True)


@pytest.mark.parametrize("name", ["c5_shards2", "c5_shards4"])
def test_sharded_oracle_equals_unsharded(oracle, name):
    """The shard protocol loses nothing: same ids/top-k as the whole-row path at cap 64."""
    case = CASES[name]
    x, p, u = _inputs(case)
    whole, wids, wvals = oracle.sample_rows(x, p, u, 64)
    for r, e in enumerate(case["expected"]):
        n = e["pool_size"]
        assert int(whole[r]["id"]) == e["id"]
        assert list(wids[r, :n]) == e["topk_ids"]
        assert float(whole[r]["sum_exp"]) == pytest.approx(e["sum_exp"], rel=REL)
        assert float(whole[r]["probability"]) == pytest.approx(e["probability"], rel=REL)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_matches_golden(name):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200._lib import OUTCOME_DTYPE, check, lib
    from tabby_b200 import Sampler
    from tabby_b200.sharded import BLOCK_WORDS, SHARD_TOP_K

    case = CASES[name]
    x, p, u = _inputs(case)
    rows, V = x.shape
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    pd = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    cap = case["cap"]
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ids = torch.full((rows, cap), -1, dtype=torch.int32, device=dev)
    vals = torch.zeros((rows, cap), dtype=torch.float32, device=dev)
    L = lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with Sampler(0, max_top_k=cap, max_rows=rows, max_vocab=V) as s:
        if case["shards"]:
            P = case["shards"]
            blocks = torch.empty((P * rows, BLOCK_WORDS), dtype=torch.float32, device=dev)
            for sh in range(P):
                lo, hi = sh * V // P, (sh + 1) * V // P
                part = xd[:, lo:hi]
                check(L.tabby_shard_local_async(
                    s.handle, part.data_ptr(), xd.stride(0), rows, hi - lo, lo,
                    blocks[sh * rows].data_ptr(), BLOCK_WORDS, stream))
            check(L.tabby_shard_merge_async(
                s.handle, blocks.data_ptr(), P, rows, BLOCK_WORDS, pd.data_ptr(), ud.data_ptr(),
                out.data_ptr(), ids.data_ptr(), vals.data_ptr(), SHARD_TOP_K, stream))
        else:
            check(L.tabby_sample_rows_async(
                s.handle, xd.data_ptr(), V, rows, V, pd.data_ptr(), ud.data_ptr(),
                out.data_ptr(), ids.data_ptr(), vals.data_ptr(), cap, stream))
        torch.cuda.synchronize()
    _check(case, out.cpu().numpy().view(OUTCOME_DTYPE), ids.cpu().numpy(), vals.cpu().numpy(),
           exact_floats=False)
