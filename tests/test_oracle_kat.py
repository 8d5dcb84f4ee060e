"""CPU: the parity oracle pinned against the reference's own known answers.

The reference has no golden vectors for the sampling path (its model-driven GPU tests
need weights that are not in the repository); what it does pin is the host-side
arithmetic in tests/sampling.test.ts:206-250 ("sampling maths", on the fixture
{maxLogit 10, sumExp 2.5, ids [1,2,3,4], logits [10,9,8,7]}), the generator of
tests/support.ts:7-16 / src/engine/sampler.ts:105-119, and the exact CPU top-k order of
src/engine/sampler.ts:26-30. Every check here runs on three implementations:

* ``py``      a plain-Python restatement written in this file (sampler.ts:147-212 with
              math.exp), independent of the C code;
* ``oracle``  the C restatement under oracle/ (fdlibm-method exp, as V8 evaluates);
* ``lib``     the product library's host entry tabby_sample_from_topk, which runs the
              same float64 finalize code the GPU kernel runs.
"""
import math

import numpy as np
import pytest

FIXTURE = dict(maxLogit=10.0, sumExp=2.5, ids=[1, 2, 3, 4], logits=[10.0, 9.0, 8.0, 7.0])
M32 = 0xFFFFFFFF


# --- independent plain-Python restatements ----------------------------------------------
def py_mulberry32(seed):
    """tests/support.ts:7-16."""
    a = seed & M32

    def nxt():
        nonlocal a
        a = (a + 0x6D2B79F5) & M32
        t = a
        t = ((t ^ (t >> 15)) * (t | 1)) & M32
        t ^= (t + (((t ^ (t >> 7)) * (t | 61)) & M32)) & M32
        return ((t ^ (t >> 14)) & M32) / 4294967296

    return nxt


def py_sample_from_topk(top, temperature, top_p, u):
    """sampler.ts:147-212 line by line, Python floats (IEEE doubles) and math.exp."""
    ids, logits = top["ids"], top["logits"]
    if not ids:
        raise ValueError("sampleFromTopK: empty candidate set")
    m, s = top["maxLogit"], top["sumExp"]
    exact = [math.exp(l - m) / s for l in logits]
    pool_mass = 0.0
    for e in exact:
        pool_mass += e
    if temperature <= 0:
        return dict(id=ids[0], probability=exact[0], consideredCount=1, poolMass=pool_mass,
                    poolExhausted=False)
    scaled = [math.exp((l - m) / temperature) for l in logits]
    scaled_total = 0.0
    for w in scaled:
        scaled_total += w
    weights = [w / scaled_total for w in scaled]
    cut = len(ids)
    exhausted = False
    if top_p < 1:
        cum = 0.0
        for i, w in enumerate(weights):
            cum += w
            if cum >= top_p:
                cut = i + 1
                break
        exhausted = pool_mass < top_p
    total = 0.0
    for w in weights[:cut]:
        total += w
    target = u * total
    running = 0.0
    chosen = cut - 1
    for i in range(cut):
        running += weights[i]
        if target < running:
            chosen = i
            break
    return dict(id=ids[chosen], probability=exact[chosen], consideredCount=cut,
                poolMass=pool_mass, poolExhausted=exhausted)


# --- the three implementations behind one call ------------------------------------------
def _oracle_impl(oracle):
    def run(top, t, p, u):
        return oracle.sample_from_topk(top["ids"], top["logits"], top["maxLogit"],
                                       top["sumExp"], t, p, u)
    return run


def _lib_impl():
    from tabby_b200 import SamplingParams, TopKResult, sample_from_topk

    class _U:
        def __init__(self, u):
            self.u = u

        def next(self):
            return self.u

    def run(top, t, p, u):
        o = sample_from_topk(TopKResult(top["maxLogit"], top["sumExp"], list(top["ids"]),
                                        list(top["logits"])),
                             SamplingParams(t, len(top["ids"]), p), _U(u))
        return dict(id=o.id, probability=o.probability, consideredCount=o.consideredCount,
                    poolMass=o.poolMass, poolExhausted=o.poolExhausted)
    return run


@pytest.fixture(params=["py", "oracle", "lib"])
def impl(request, oracle):
    if request.param == "py":
        return py_sample_from_topk
    if request.param == "oracle":
        return _oracle_impl(oracle)
    return _lib_impl()


# sampling.test.ts:216-220
def test_kat_argmax_at_temperature_zero(impl):
    o = impl(FIXTURE, 0.0, 1.0, py_mulberry32(0)())
    assert o["id"] == 1 and o["consideredCount"] == 1


# sampling.test.ts:222-227
def test_kat_top_p_narrows(impl):
    wide = impl(FIXTURE, 1.0, 1.0, py_mulberry32(0)())
    narrow = impl(FIXTURE, 1.0, 0.5, py_mulberry32(0)())
    assert 1 <= narrow["consideredCount"] < wide["consideredCount"]
    assert wide["consideredCount"] == 4 and narrow["consideredCount"] == 1


# sampling.test.ts:229-239
def test_kat_pool_exhausted(impl):
    o = impl(dict(FIXTURE, sumExp=100.0), 1.0, 0.9, py_mulberry32(0)())
    assert o["poolMass"] < 0.9 and o["poolExhausted"] is True


# sampling.test.ts:241-249
def test_kat_temperature_spreads(impl):
    nxt = py_mulberry32(12345)
    chosen = {impl(FIXTURE, 2.0, 1.0, nxt())["id"] for _ in range(200)}
    assert len(chosen) > 1


def test_kat_pool_mass_value(impl):
    o = impl(FIXTURE, 1.0, 1.0, 0.5)
    want = sum(math.exp(-i) for i in range(4)) / 2.5
    assert o["poolMass"] == pytest.approx(want, rel=1e-15)


def test_empty_candidate_set_raises(oracle):
    with pytest.raises(ValueError, match="empty candidate set"):
        py_sample_from_topk(dict(FIXTURE, ids=[], logits=[]), 1.0, 1.0, 0.5)
    with pytest.raises(ValueError, match="empty candidate set"):
        oracle.sample_from_topk([], [], 0.0, 1.0, 1.0, 1.0, 0.5)


def test_three_implementations_agree_on_random_pools(oracle):
    """Token ids, cut and flags equal; float64 outputs equal to 1e-14 (the two exp
    implementations may differ in the last bit); oracle and lib bit-identical."""
    g = np.random.default_rng(7)
    lib_run = _lib_impl()
    orc_run = _oracle_impl(oracle)
    for trial in range(300):
        n = int(g.integers(1, 80))
        vals = np.sort(g.normal(0, 3, n).astype(np.float32))[::-1]
        top = dict(maxLogit=float(vals[0]), sumExp=float(np.float32(g.uniform(1.0, 50.0))),
                   ids=[int(i) for i in g.permutation(100000)[:n]],
                   logits=[float(v) for v in vals])
        t = float(g.choice([0.0, 0.3, 0.7, 1.0, 1.5, 2.0]))
        p = float(g.choice([1.0, 0.95, 0.9, 0.5, float(g.uniform())]))
        u = float(g.uniform())
        a, b, c = py_sample_from_topk(top, t, p, u), orc_run(top, t, p, u), lib_run(top, t, p, u)
        assert b == c, (trial, b, c)
        for key in ("id", "consideredCount", "poolExhausted"):
            assert a[key] == b[key], (trial, key, a, b)
        for key in ("probability", "poolMass"):
            assert a[key] == pytest.approx(b[key], rel=1e-14, abs=0)


# --- SeededRandom ---------------------------------------------------------------------
@pytest.mark.parametrize("seed", [0, 1, 42, 12345, 0xFFFFFFFF, 2**31])
def test_mulberry32_three_ways(oracle, seed):
    from tabby_b200 import SeededRandom

    a, b, c = py_mulberry32(seed), oracle.SeededRandom(seed), SeededRandom(seed)
    for _ in range(1000):
        x = a()
        assert x == b.next() == c.next()
        assert 0.0 <= x < 1.0


def test_mulberry32_first_draws_seed0():
    # state 0x6D2B79F5 after one step; the first u32 is fixed by the integer steps alone.
    nxt = py_mulberry32(0)
    first = nxt()
    assert first == pytest.approx(0.26642920868471265, abs=0)


# --- exp, top-k, argmax, pool rule ----------------------------------------------------
def test_js_exp_within_one_ulp_of_libm(oracle):
    g = np.random.default_rng(3)
    xs = np.concatenate([g.uniform(-745, 709, 20000), g.normal(0, 3, 20000),
                         [0.0, -0.0, 1.0, -1.0, 709.78, -745.1, 1e-300, -1e-300]])
    for x in xs:
        a, b = oracle.js_exp(float(x)), math.exp(float(x))
        if b == 0.0 or math.isinf(b):
            assert a == b
        else:
            assert abs(a - b) <= math.ulp(b), (x, a, b)
    assert math.isnan(oracle.js_exp(float("nan")))
    assert oracle.js_exp(float("inf")) == float("inf")
    assert oracle.js_exp(float("-inf")) == 0.0


def _np_topk(row, k):
    order = np.lexsort((np.arange(row.size), -row.astype(np.float64)))
    return order[:k]


@pytest.mark.parametrize("k", [1, 2, 8, 40, 64, 1024])  # sampling.test.ts:85-94, plus 1024
def test_oracle_topk_matches_full_sort(oracle, k):
    g = np.random.default_rng(k)
    row = np.round(g.normal(0, 2, 49152)).astype(np.float32)  # heavy ties
    ids, vals = oracle.topk(row, k)
    want = _np_topk(row, k)
    np.testing.assert_array_equal(ids, want)
    np.testing.assert_array_equal(vals, row[want])


def test_oracle_argmax_lowest_index_on_ties(oracle):
    row = np.zeros(1000, np.float32)
    row[[17, 400, 999]] = 5.0
    assert oracle.argmax(row) == 17
    assert oracle.topk(row, 1)[0][0] == 17


def test_oracle_signed_zeros_tie_on_the_index(oracle):
    """sampler.ts:28 sorts by `b.value - a.value || a.id - b.id`: +0 and -0 differ by 0,
    so they tie and the lower id comes first; the values keep their sign bits."""
    row = np.full(64, -1.0, np.float32)
    row[[5, 9, 40]] = [-0.0, 0.0, -0.0]
    ids, vals = oracle.topk(row, 4)
    np.testing.assert_array_equal(ids, [5, 9, 40, 0])
    np.testing.assert_array_equal(np.asarray(vals, np.float32).view(np.uint32),
                                  np.array([-0.0, 0.0, -0.0, -1.0], np.float32).view(np.uint32))
    assert oracle.argmax(row) == 5  # strictly greater scan: -0 is not above +0


@pytest.mark.parametrize("t,k,cap,want", [
    (0.0, 40, 64, 1), (-1.0, 0, 64, 1), (0.7, 0, 64, 64), (0.7, 40, 64, 40),
    (0.7, 100, 64, 64), (0.7, -5, 64, 1), (1.0, 0, 1024, 1024), (1.0, 1000, 1024, 1000),
])
def test_pool_rule(oracle, t, k, cap, want):
    """inference.worker.ts:120-123: T<=0 -> 1, else min(cap, max(1, topK || cap))."""
    from tabby_b200 import pool_size

    assert oracle.pool_size(t, k, cap) == want
    assert pool_size(t, k, cap) == want


# --- generator consumption: greedy calls do not draw ------------------------------------
def py_sample_from_topk_rng(top, temperature, top_p, nxt):
    """sampleFromTopK(top, params, random) as sampler.ts:147-212 calls random.next(): once,
    after the greedy return (:159-167), at :194."""
    if temperature <= 0:
        return py_sample_from_topk(top, temperature, top_p, 0.0)
    return py_sample_from_topk(top, temperature, top_p, nxt())


def test_greedy_call_leaves_the_generator_alone(oracle):
    """T=0 call, then T=1 call, then a bare next(): the reference's first draw goes to the
    T=1 call and the second to the bare next(). The Python mirror, the oracle and the
    library's host entry must agree id for id and leave the same generator state."""
    from tabby_b200 import SamplingParams, SeededRandom, sample_from_topk
    from tabby_b200.sampler import TopKResult

    top = TopKResult(FIXTURE["maxLogit"], FIXTURE["sumExp"], FIXTURE["ids"],
                     FIXTURE["logits"])
    for seed in (0, 7, 12345):
        nxt = py_mulberry32(seed)
        want = [py_sample_from_topk_rng(FIXTURE, 0.0, 1.0, nxt)["id"],
                py_sample_from_topk_rng(FIXTURE, 1.0, 1.0, nxt)["id"]]
        want_next = nxt()

        ro = oracle.SeededRandom(seed)
        got_or = []
        for t in (0.0, 1.0):
            u = ro.next() if t > 0 else 0.0
            got_or.append(oracle.sample_from_topk(FIXTURE["ids"], FIXTURE["logits"],
                                                  FIXTURE["maxLogit"], FIXTURE["sumExp"],
                                                  t, 1.0, u)["id"])
        rl = SeededRandom(seed)
        got_lib = [sample_from_topk(top, SamplingParams(t, 4, 1.0), rl).id for t in (0.0, 1.0)]
        assert got_lib == want and got_or == want, (seed, want, got_or, got_lib)
        assert rl.next() == want_next == ro.next()


def test_batch_uniforms_draw_only_for_sampling_rows():
    """Sampler's per-row uniforms from one SeededRandom: rows in order, a draw only where
    sampleFromTopK draws (temperature > 0), the same rule as the device-RNG entry."""
    from tabby_b200 import SeededRandom
    from tabby_b200.sampler import Sampler, params_array, SamplingParams

    temps = [0.0, 0.7, 0.0, 1.3, -1.0, 0.2]
    p = params_array([SamplingParams(t, 40, 0.9) for t in temps], len(temps))
    rng = SeededRandom(99)
    u = Sampler._uniforms(len(temps), rng, p)
    nxt = py_mulberry32(99)
    want = [nxt() if t > 0 else 0.0 for t in temps]
    assert list(u) == want
    assert rng.next() == nxt()


# --- exact decision boundaries -------------------------------------------------------
# Pools of m equal logits at the row maximum have weights of exactly 1/m (m a power of
# two), so the cumulative sums hit top_p and u * total exactly. sampler.ts:181 keeps the
# first i with cumulative >= topP and :199 the first i with target < running: these
# cases pin both comparisons on the three implementations. Cases are (m, T, top_p, u,
# expected cut, expected chosen index).
BOUNDARY_CASES = [
    (4, 1.0, 0.5, 0.5, 2, 1),      # cumulative == topP at i=1; target == running at i=0
    (4, 1.0, 1.0, 0.25, 4, 1),     # no nucleus; target == cum[0]
    (4, 0.7, 0.75, 0.0, 3, 0),     # u = 0 takes the first candidate
    (2, 1.0, 0.5, 0.9999999, 1, 0),
    (4, 1.0, 0.5000000000000001, 0.5, 3, 1),  # topP one ulp above cum[1]
    (4, 1.0, 1.0, 1.0 - 2.0 ** -53, 4, 3),    # largest u below 1: the last candidate
    (8, 1.3, 0.375, 2.0 / 3.0, 3, 2),  # target rounds to 0.25 == cum[1]
    (128, 1.0, 0.5, 0.5, 64, 32),  # target == cum[31]
]


def boundary_pool(m):
    return dict(maxLogit=4.0, sumExp=float(m), ids=[3 * i + 1 for i in range(m)],
                logits=[4.0] * m)


@pytest.mark.parametrize("case", BOUNDARY_CASES)
def test_exact_boundaries_three_ways(oracle, case):
    m, t, p, u, cut, chosen = case
    top = boundary_pool(m)
    a = py_sample_from_topk(top, t, p, u)
    assert (a["consideredCount"], a["id"]) == (cut, top["ids"][chosen]), a
    b, c = _oracle_impl(oracle)(top, t, p, u), _lib_impl()(top, t, p, u)
    assert a == b == c
