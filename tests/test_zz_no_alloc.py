"""The allocation-free entry point tabby_sample_rows_noalloc.

Callers that cannot call cudaMalloc (code under an allocator that owns all device
memory, plug-in hosts that forbid allocation on their request path) sample through this
entry point; its scratch lives in a fixed device array inside the library. This test
calls it through the C ABI and checks it against the handle-based entry point
tabby_sample_rows_async on the same inputs, twice in a row (the second call sees the
array as the first left it). It runs last so a failure here never hides the others,
and it passes alone in a fresh process as well as after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu

REL = 1e-5  # same tolerance as the parity tests for float outputs


def _run(torch, fn, x, p, u, cap):
    from tabby_b200._lib import OUTCOME_DTYPE

    rows, vocab = x.shape
    dev = torch.device("cuda", 0)
    logits = torch.from_numpy(x).to(dev)
    pd = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ids = torch.full((rows, cap), -1, dtype=torch.int32, device=dev)
    vals = torch.zeros((rows, cap), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    fn(logits, pd, ud, out, ids, vals, stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(OUTCOME_DTYPE), ids.cpu().numpy(), vals.cpu().numpy()


def _same(a, b):
    (oa, ia, va), (ob, ib, vb) = a, b
    assert (oa["status"] == 0).all() and (ob["status"] == 0).all()
    np.testing.assert_array_equal(oa["id"], ob["id"])
    np.testing.assert_array_equal(oa["considered_count"], ob["considered_count"])
    np.testing.assert_array_equal(oa["pool_size"], ob["pool_size"])
    for r in range(oa.shape[0]):
        k = int(oa["pool_size"][r])
        np.testing.assert_array_equal(ia[r, :k], ib[r, :k])
        np.testing.assert_array_equal(va[r, :k], vb[r, :k])
    np.testing.assert_allclose(oa["probability"], ob["probability"], rtol=REL)
    np.testing.assert_allclose(oa["pool_mass"], ob["pool_mass"], rtol=REL)
    np.testing.assert_allclose(oa["sum_exp"], ob["sum_exp"], rtol=REL)


def test_noalloc_matches_handle_entry_point_twice():
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import check, lib

    L = lib()
    cap = 256
    sampler = Sampler(0, max_top_k=cap, max_rows=128, max_vocab=151936)

    def with_handle(logits, pd, ud, out, ids, vals, stream):
        rows, vocab = logits.shape
        check(L.tabby_sample_rows_async(sampler.handle, logits.data_ptr(), vocab, rows, vocab,
                                        pd.data_ptr(), ud.data_ptr(), out.data_ptr(),
                                        ids.data_ptr(), vals.data_ptr(), cap, stream))

    def without_alloc(logits, pd, ud, out, ids, vals, stream):
        rows, vocab = logits.shape
        check(L.tabby_sample_rows_noalloc(logits.data_ptr(), vocab, rows, vocab, cap,
                                          pd.data_ptr(), ud.data_ptr(), out.data_ptr(),
                                          ids.data_ptr(), vals.data_ptr(), cap, stream))

    # Small batches split every row into slices, so the scratch array is really used; the
    # 100-row call runs as four launches over the same array (32 rows a launch).
    from oracle import oracle as orc

    for call, (rows, seed) in enumerate([(8, 1), (5, 2), (100, 3)]):
        x, p, u = synth.config("c4", seed=seed, rows=rows)
        p["top_k"] = np.resize(np.array([0, 20, 100, 256, 1, 40, 7, 200]), rows)
        a = _run(torch, without_alloc, x, p, u, cap)
        b = _run(torch, with_handle, x, p, u, cap)
        _same(a, b)
        ref, rids, rvals = orc.sample_rows(x, p, u, cap)
        np.testing.assert_array_equal(a[0]["id"], ref["id"])
        for r in range(rows):
            k = int(ref[r]["pool_size"])
            np.testing.assert_array_equal(a[1][r, :k], rids[r, :k])
        np.testing.assert_allclose(a[0]["probability"], ref["probability"], rtol=REL)
    sampler.close()


def test_noalloc_rejects_sizes_beyond_its_limit():
    if not gpu_available():
        pytest.skip("no CUDA device")
    from tabby_b200._lib import TABBY_EINVAL, TABBY_NOALLOC_MAX_TOP_K, lib

    L = lib()
    rc = L.tabby_sample_rows_noalloc(ctypes.c_void_p(16), 100, 1, 100,
                                     TABBY_NOALLOC_MAX_TOP_K + 1, ctypes.c_void_p(16),
                                     ctypes.c_void_p(16), ctypes.c_void_p(16), None, None, 0, None)
    assert rc == TABBY_EINVAL
    assert b"limit" in L.tabby_last_error()
