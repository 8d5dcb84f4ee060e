"""GPU parity: the CUDA sampler (through the C ABI) against the CPU oracle.

Bar: bit-exact token ids, top-k id sets, their order and their logits (ties -> lower
index, as sampler.ts:28 and topk_partial.wgsl:40-42); considered_count exact; float
outputs (sumExp, probability, poolMass) within 1e-5 relative.
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu

REL = 1e-5  # tolerance north_star states for normalised probabilities


@pytest.fixture(scope="module")
def torch_cuda():
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    return torch


_SAMPLERS = {}


def sampler(cap):
    from tabby_b200 import Sampler

    if cap not in _SAMPLERS:
        _SAMPLERS[cap] = Sampler(0, max_top_k=cap, max_rows=512, max_vocab=151936)
    return _SAMPLERS[cap]


def run_gpu(torch, x, params, u, cap, stride=None, offset=0):
    """Run tabby_sample_rows_async on x (rows, vocab); optional padded row stride and
    element offset of the first row (to exercise misaligned TMA heads)."""
    from tabby_b200._lib import OUTCOME_DTYPE

    rows, vocab = x.shape
    stride = stride or vocab
    buf = torch.zeros(offset + rows * stride + 8, dtype=torch.float32)
    view = buf[offset:offset + rows * stride].view(rows, stride)
    view[:, :vocab] = torch.from_numpy(x)
    dev = buf.cuda()
    logits = dev[offset:offset + rows * stride].view(rows, stride)[:, :vocab]
    p = torch.from_numpy(params.view(np.uint8).copy()).cuda()
    ud = torch.from_numpy(np.ascontiguousarray(u, np.float64)).cuda()
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device="cuda")
    ids = torch.full((rows, cap), -1, dtype=torch.int32, device="cuda")
    vals = torch.zeros((rows, cap), dtype=torch.float32, device="cuda")
    s = sampler(cap)
    s.sample_rows_async(logits, p, ud, out, ids, vals)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(OUTCOME_DTYPE), ids.cpu().numpy(), vals.cpu().numpy()


def assert_parity(oracle, x, params, u, cap, got, check_finalize=True):
    out, ids, vals = got
    ref, rids, rvals = oracle.sample_rows(x, params, u, cap)
    rows = x.shape[0]
    for r in range(rows):
        o, e = out[r], ref[r]
        assert o["status"] == 0, f"row {r}: status {o['status']}"
        k = int(e["pool_size"])
        assert int(o["pool_size"]) == k, f"row {r}: pool {o['pool_size']} vs {k}"
        np.testing.assert_array_equal(ids[r, :k], rids[r, :k], err_msg=f"row {r} top-k ids")
        np.testing.assert_array_equal(vals[r, :k].view(np.uint32), rvals[r, :k].view(np.uint32),
                                      err_msg=f"row {r} top-k logits")
        assert np.float32(o["max_logit"]).view(np.uint32) == np.float32(e["max_logit"]).view(
            np.uint32), f"row {r} maxLogit"
        assert abs(float(o["sum_exp"]) - float(e["sum_exp"])) <= REL * float(e["sum_exp"]), (
            f"row {r} sumExp {o['sum_exp']} vs {e['sum_exp']}")
        assert int(o["id"]) == int(e["id"]), f"row {r}: id {o['id']} vs {e['id']}"
        assert int(o["considered_count"]) == int(e["considered_count"]), f"row {r} count"
        assert abs(o["probability"] - e["probability"]) <= REL * e["probability"] + 1e-300
        assert abs(o["pool_mass"] - e["pool_mass"]) <= REL * e["pool_mass"]
        tp = float(params["top_p"][r])
        if abs(float(e["pool_mass"]) - tp) > 1e-4:
            assert int(o["pool_exhausted"]) == int(e["pool_exhausted"]), f"row {r} exhausted"
        if check_finalize:
            # The device finalize is the reference's float64 arithmetic: fed the GPU's own
            # TopKResult, the oracle's sampleFromTopK reproduces every output bit.
            fo = oracle.sample_from_topk(ids[r, :k], vals[r, :k], o["max_logit"], o["sum_exp"],
                                         params["temperature"][r], params["top_p"][r], u[r])
            assert fo["id"] == int(o["id"])
            assert fo["consideredCount"] == int(o["considered_count"])
            assert fo["probability"] == float(o["probability"])
            # poolMass comes from a parallel float64 sum unless the sequential replay ran.
            assert abs(fo["poolMass"] - float(o["pool_mass"])) <= 1e-12 * fo["poolMass"]
            assert fo["poolExhausted"] == bool(o["pool_exhausted"])


@pytest.mark.parametrize("cap", [64, 1024])
def test_c1_single_row(torch_cuda, oracle, cap):
    from tabby_b200 import synth

    for seed in range(4):
        x, p, u = synth.config("c1", seed=seed)
        assert_parity(oracle, x, p, u, cap, run_gpu(torch_cuda, x, p, u, cap))


@pytest.mark.parametrize("k", [1, 50])
def test_c2_tie_heavy(torch_cuda, oracle, k):
    from tabby_b200 import synth

    for seed in range(4):
        x, p, u = synth.config("c2", seed=seed, top_k=k)
        got = run_gpu(torch_cuda, x, p, u, 64)
        assert_parity(oracle, x, p, u, 64, got)
        # Greedy/argmax: the lowest index among the 8 forced maxima.
        assert got[1][0, 0] == oracle.argmax(x[0])


@pytest.mark.parametrize("k", [1, 8, 64, 256, 1024])
def test_c3_long_tail_sweep(torch_cuda, oracle, k):
    from tabby_b200 import synth

    x, p, u = synth.config("c3", seed=1, rows=16, top_k=k)
    assert_parity(oracle, x, p, u, 1024, run_gpu(torch_cuda, x, p, u, 1024))


def test_c4_heterogeneous(torch_cuda, oracle):
    from tabby_b200 import synth

    x, p, u = synth.config("c4", seed=2, rows=64)
    assert_parity(oracle, x, p, u, 1024, run_gpu(torch_cuda, x, p, u, 1024))


def test_c4_full_batch(torch_cuda, oracle):
    from tabby_b200 import synth

    x, p, u = synth.config("c4", seed=3)
    assert_parity(oracle, x, p, u, 1024, run_gpu(torch_cuda, x, p, u, 1024), check_finalize=False)


@pytest.mark.parametrize("vocab", [1, 3, 5, 17, 300, 1001, 4099, 49153])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_ragged_sizes_and_alignment(torch_cuda, oracle, vocab, offset):
    """Vocab not a multiple of 4 and rows starting off a 16-byte boundary: the TMA bulk
    copy covers the aligned middle, plain loads the ragged ends."""
    g = np.random.default_rng(vocab * 10 + offset)
    rows = 3
    x = (3 * g.standard_normal((rows, vocab))).astype(np.float32)
    p = oracle.make_params([0.9, 0.0, 1.3], [0.95, 1.0, 0.5], [40, 1, 0], rows)
    u = g.random(rows)
    stride = vocab + 5
    got = run_gpu(torch_cuda, x, p, u, 64, stride=stride, offset=offset)
    assert_parity(oracle, x, p, u, 64, got)


def test_all_equal_row_takes_lowest_indices(torch_cuda, oracle):
    """151936 exact ties: the exact-threshold path must take the k lowest indices."""
    rows, vocab = 2, 151936
    x = np.zeros((rows, vocab), np.float32)
    x[1] = 1.5
    p = oracle.make_params(1.0, 1.0, 50, rows)
    u = np.array([0.3, 0.9])
    out, ids, vals = run_gpu(torch_cuda, x, p, u, 64)
    np.testing.assert_array_equal(ids[:, :50], np.tile(np.arange(50), (2, 1)))
    assert_parity(oracle, x, p, u, 64, (out, ids, vals))


def test_ties_straddling_the_kth(torch_cuda, oracle):
    """Many duplicates of the k-th value spread over all CTAs of the cluster."""
    g = np.random.default_rng(5)
    rows, vocab = 4, 151936
    x = np.round(g.standard_normal((rows, vocab)) * 2).astype(np.float32)  # ~9 distinct values
    for k, cap in [(1, 64), (40, 64), (1000, 1024)]:
        p = oracle.make_params(1.0, 1.0, k, rows)
        u = g.random(rows)
        assert_parity(oracle, x, p, u, cap, run_gpu(torch_cuda, x, p, u, cap))


def test_signed_zero_and_negative_values(torch_cuda, oracle):
    rows, vocab = 3, 5000
    g = np.random.default_rng(9)
    x = -np.abs(g.standard_normal((rows, vocab))).astype(np.float32)
    x[0, [10, 20, 30]] = [-0.0, 0.0, -0.0]
    x[1, :] = -0.0
    x[1, 7] = 0.0
    x[2] = -1e30
    p = oracle.make_params(0.7, 0.9, 40, rows)
    u = g.random(rows)
    out, ids, vals = run_gpu(torch_cuda, x, p, u, 64)
    assert_parity(oracle, x, p, u, 64, (out, ids, vals))
    assert ids[1, 0] == 0 and np.signbit(vals[1, 0])  # -0 at index 0 ties +0 at 7


def test_k_larger_than_vocab(torch_cuda, oracle):
    x = np.array([[3.0, 1.0, 2.0, 2.0, -1.0]], np.float32)
    p = oracle.make_params(1.0, 1.0, 0, 1)
    u = np.array([0.99])
    out, ids, vals = run_gpu(torch_cuda, x, p, u, 64)
    assert out[0]["pool_size"] == 5
    assert_parity(oracle, x, p, u, 64, (out, ids, vals))


def test_bad_logits_are_reported_per_row(torch_cuda, oracle):
    from tabby_b200._lib import TABBY_EINPUT, TABBY_OK

    rows, vocab = 4, 2000
    x = np.zeros((rows, vocab), np.float32)
    x[1, 5] = np.nan
    x[2, 1999] = np.inf
    x[3, 0] = -3.0e38
    p = oracle.make_params(1.0, 1.0, 10, rows)
    out, _, _ = run_gpu(torch_cuda, x, p, np.zeros(rows), 64)
    assert list(out["status"]) == [TABBY_OK, TABBY_EINPUT, TABBY_EINPUT, TABBY_EINPUT]


def test_batch_sweep_cluster_sizes(torch_cuda, oracle):
    """B in {1..256} picks clusters of 16, 8 (and the geometry for small vocabularies)."""
    from tabby_b200 import synth

    for rows in [1, 2, 7, 37, 150]:
        x, p, u = synth.config("c4", seed=rows, rows=rows)
        assert_parity(oracle, x, p, u, 1024, run_gpu(torch_cuda, x, p, u, 1024),
                      check_finalize=False)


def test_topk_block_wire_format(torch_cuda, oracle):
    """tabby_topk_rows_async == ForwardPass.runFull(ids, {topK}) block (forward.ts:126-157)."""
    from tabby_b200 import Sampler, decode_sample_block, synth

    s = sampler(64)
    x, _, _ = synth.config("c1", seed=11, rows=3)
    t = torch_cuda.from_numpy(x).cuda()
    for k in [0, 1, 2, 8, 40, 64]:
        blk = s.topk_block(t, k).cpu().numpy()
        for r in range(3):
            top = decode_sample_block(blk[r], k)
            rid, rv = oracle.topk(x[r], k)
            assert top.ids == list(rid)
            assert top.logits == [float(v) for v in rv]
            assert top.maxLogit == float(oracle.row_max(x[r]))
            se = oracle.sum_exp_f64(x[r], oracle.row_max(x[r]))
            assert abs(top.sumExp - se) <= REL * se
    with pytest.raises(Exception, match="topK"):
        s.topk_block(t, 65)


def test_sample_api_host_and_device(torch_cuda, oracle):
    """sample(logits, {temperature, topK, topP}, rng): the drop-in call, host buffers
    (copies inside the library) and device tensors give the oracle's token."""
    from tabby_b200 import SamplingParams, SeededRandom, synth

    s = sampler(64)
    x, _, _ = synth.config("c1", seed=21, rows=1)
    params = SamplingParams(temperature=0.8, topK=40, topP=0.95, seed=42)
    rid, rv = oracle.topk(x[0], 40)
    mx = oracle.row_max(x[0])
    se = np.float32(oracle.sum_exp_f64(x[0], mx))
    for i in range(3):
        u = SeededRandom(42 + i).next()
        ref = oracle.sample_from_topk(rid, rv, mx, se, 0.8, 0.95, u)
        assert s.sample(x, params, SeededRandom(42 + i)) == ref["id"]
        assert s.sample(torch_cuda.from_numpy(x).cuda(), params, SeededRandom(42 + i)) == ref["id"]


def test_seeded_determinism(torch_cuda):
    """Same seed replays, another seed diverges (sampling.test.ts:151-204)."""
    from tabby_b200 import SamplingParams, SeededRandom, synth

    s = sampler(64)
    x, _, _ = synth.config("c1", seed=3, rows=24)
    t = torch_cuda.from_numpy(x).cuda()
    p = SamplingParams(0.9, 40, 0.95)
    a = s.sample_batch(t, p, SeededRandom(42)).ids
    b = s.sample_batch(t, p, SeededRandom(42)).ids
    c = s.sample_batch(t, p, SeededRandom(43)).ids
    np.testing.assert_array_equal(a, b)
    assert (a != c).any()
    g0 = s.sample_batch(t, SamplingParams(0, 1, 1), SeededRandom(1)).ids
    g1 = s.sample_batch(t, SamplingParams(0, 1, 1), SeededRandom(999)).ids
    np.testing.assert_array_equal(g0, g1)


@pytest.mark.parametrize("rows", [2, 256])
def test_threshold_estimate_failures(torch_cuda, oracle, rows):
    """Rows built so the threshold estimated from the plan's sample (512 float4 groups in
    32 runs of 16 spread over the row) is wrong in both directions: too high (the sampled
    groups hold the largest logits, so fewer than k logits pass) and too low (they hold the
    smallest, so the candidates overflow the row's list). Both must end in the exact result
    through the re-filter. Small batches split rows into chunks (plan sample); 256 rows are
    taken whole (the first iteration of every warp is the sample): both layouts are marked."""
    g = np.random.default_rng(17)
    vocab = 151936
    ngroups = vocab // 4
    sampled = np.zeros(vocab, bool)
    for run in range(32):
        start = min(max((2 * run + 1) * ngroups // 64 - 8, 0), ngroups - 16)
        sampled[4 * start:4 * (start + 16)] = True
    # Whole rows (256 rows a launch) sample the first 128 groups of each warp's 16th.
    seg = (ngroups + 15) // 16
    for w in range(16):
        sampled[4 * w * seg:4 * min(w * seg + 128, ngroups)] = True
    x = g.standard_normal((rows, vocab)).astype(np.float32)
    x[0::2, sampled] += 20.0   # too-high estimate
    x[1::2, sampled] -= 20.0   # too-low estimate
    for k, cap in [(1, 64), (50, 64), (1000, 1024)]:
        p = oracle.make_params(1.0, 0.9, k, rows)
        u = g.random(rows)
        assert_parity(oracle, x, p, u, cap, run_gpu(torch_cuda, x, p, u, cap))
