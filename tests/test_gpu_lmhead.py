"""GPU: the fused LM head (tcgen05 GEMM with the sampling pass as its epilogue) against an
fp32 GEMM of the same bf16 inputs and the CPU oracle.

The logits the epilogue saw (the test-only d_logits_out) must equal torch's fp32 product
of the bf16 hidden states and weights within 1e-4 (fp32 accumulation in a different
order); the sampled tokens, the top-k ids, order and logits must be bit-exact against the
oracle run on those logits, and probability / sumExp within 1e-5 relative. The fused call
without d_logits_out must give the same outcomes.
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu

REL = 1e-5
CAP = 64  # the fused path's pool cap: the reference's MAX_TOP_K


def _run(torch, h, w, p, u, want_logits):
    from tabby_b200._lib import OUTCOME_DTYPE, check, lib

    L = lib()
    rows, hidden = h.shape
    vocab = w.shape[0]
    handle = __import__("ctypes").c_void_p()
    check(L.tabby_lmhead_create(0, max(rows, 1), vocab, hidden, __import__("ctypes").byref(handle)))
    pd = torch.from_numpy(p.view(np.uint8).copy()).cuda()
    ud = torch.from_numpy(u).cuda()
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device="cuda")
    ids = torch.full((rows, CAP), -1, dtype=torch.int32, device="cuda")
    vals = torch.zeros((rows, CAP), dtype=torch.float32, device="cuda")
    lo = torch.zeros((rows, vocab), dtype=torch.float32, device="cuda") if want_logits else None
    check(L.tabby_lmhead_sample_async(handle, h.data_ptr(), w.data_ptr(), rows, pd.data_ptr(),
                                      ud.data_ptr(), out.data_ptr(), ids.data_ptr(),
                                      vals.data_ptr(), CAP,
                                      lo.data_ptr() if lo is not None else None,
                                      torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    L.tabby_lmhead_destroy(handle)
    return (out.cpu().numpy().view(OUTCOME_DTYPE), ids.cpu().numpy(), vals.cpu().numpy(),
            lo.cpu().numpy() if lo is not None else None)


@pytest.mark.parametrize("rows,vocab,hidden", [(1, 151936, 896), (8, 151936, 896),
                                               (64, 49152, 960), (128, 1000, 64),
                                               (37, 50003, 1024)])
def test_lmhead_matches_fp32_gemm_and_oracle(oracle, rows, vocab, hidden):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    g = torch.Generator().manual_seed(rows * 1000 + vocab)
    h = torch.randn(rows, hidden, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(vocab, hidden, generator=g) * (3.0 / hidden ** 0.5)).to(torch.bfloat16).cuda()
    rng = np.random.default_rng(rows + vocab)
    p = oracle.make_params(rng.uniform(0.3, 1.5, rows), rng.uniform(0.5, 1.0, rows),
                           rng.choice([0, 1, 20, 40, 64], rows), rows)
    p["temperature"][:: 5] = 0.0  # some greedy rows
    u = rng.random(rows)
    out, ids, vals, logits = _run(torch, h, w, p, u, True)
    ref_logits = (h.float() @ w.float().T).cpu().numpy()
    np.testing.assert_allclose(logits, ref_logits, rtol=1e-4, atol=1e-4)
    ref, rids, rvals = oracle.sample_rows(logits, p, u, CAP)
    for r in range(rows):
        o, e = out[r], ref[r]
        assert o["status"] == 0, (r, o["status"])
        k = int(e["pool_size"])
        assert int(o["pool_size"]) == k
        np.testing.assert_array_equal(ids[r, :k], rids[r, :k])
        np.testing.assert_array_equal(vals[r, :k].view(np.uint32), rvals[r, :k].view(np.uint32))
        assert int(o["id"]) == int(e["id"]), r
        assert int(o["considered_count"]) == int(e["considered_count"])
        assert abs(float(o["sum_exp"]) - float(e["sum_exp"])) <= REL * float(e["sum_exp"])
        assert abs(o["probability"] - e["probability"]) <= REL * e["probability"]
    # The production call (no logits written) gives the same outcomes, bit for bit: the
    # statistics are combined in a fixed order whichever CTA took which tile.
    out2, ids2, _, _ = _run(torch, h, w, p, u, False)
    np.testing.assert_array_equal(out2.view(np.uint8), out.view(np.uint8))
    np.testing.assert_array_equal(ids2, ids)


@pytest.mark.parametrize("rows,vocab,hidden", [(4, 151936, 896), (64, 151936, 896)])
def test_lmhead_concentrated_top_runs_exact_pass(oracle, rows, vocab, hidden):
    """Every row's best logits lie in one CTA's columns (so the fast pass's 16 a part cannot
    settle the row and the exact pass recomputes it), with tied logits among them."""
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    g = torch.Generator().manual_seed(rows * 7 + 1)
    h = torch.randn(rows, hidden, generator=g)
    w = torch.randn(vocab, hidden, generator=g) * (3.0 / hidden ** 0.5)
    for r in range(rows):
        base = 5000 + 1024 * r
        w[base:base + 100] = h[r] * (0.02 + 0.01 * torch.rand(100, 1, generator=g))
        w[base + 100:base + 110] = w[base]  # ties with id base: the lower id ranks first
    h = h.to(torch.bfloat16).cuda()
    w = w.to(torch.bfloat16).cuda()
    rng = np.random.default_rng(rows)
    p = oracle.make_params(rng.uniform(0.3, 1.5, rows), rng.uniform(0.5, 1.0, rows),
                           rng.choice([0, 40, 64], rows), rows)
    u = rng.random(rows)
    out, ids, vals, logits = _run(torch, h, w, p, u, True)
    ref, rids, rvals = oracle.sample_rows(logits, p, u, CAP)
    for r in range(rows):
        o, e = out[r], ref[r]
        assert o["status"] == 0, (r, o["status"])
        k = int(e["pool_size"])
        assert int(o["pool_size"]) == k
        np.testing.assert_array_equal(ids[r, :k], rids[r, :k])
        np.testing.assert_array_equal(vals[r, :k].view(np.uint32), rvals[r, :k].view(np.uint32))
        assert int(o["id"]) == int(e["id"]), r
        assert abs(o["probability"] - e["probability"]) <= REL * e["probability"]
