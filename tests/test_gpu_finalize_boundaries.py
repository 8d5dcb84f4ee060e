"""GPU parity where sampleFromTopK's decisions sit exactly on a boundary.

Each row holds m equal logits at its maximum (m a power of two) and the rest far below,
with top_k = m, so the pool's weights are exactly 1/m and the cumulative sums meet top_p
(sampler.ts:181, `cumulative >= topP`) or u * total (sampler.ts:199, `target < running`)
exactly. The device's parallel estimates then have no margin over their error bound, so
the finalize must replay the reference's sequential float64 arithmetic: the test checks
the outcomes against the oracle and that the replay made the decision (the outcome's
`reserved` word is 1). Runs in whole-row mode (V=4096) and chunked mode (V=49152).
"""
import numpy as np
import pytest

from tests.test_gpu_parity import assert_parity, run_gpu, torch_cuda  # noqa: F401
from tests.test_oracle_kat import BOUNDARY_CASES

pytestmark = pytest.mark.gpu


def boundary_rows(vocab, cases, seed):
    """Rows for `cases` (m, T, top_p, u, ...): m logits of 4.0 at random positions, the
    rest uniform in [-30, -20]."""
    from tabby_b200._lib import PARAMS_DTYPE

    g = np.random.default_rng(seed)
    rows = len(cases)
    x = g.uniform(-30.0, -20.0, (rows, vocab)).astype(np.float32)
    params = np.zeros(rows, PARAMS_DTYPE)
    u = np.zeros(rows, np.float64)
    for r, (m, t, p, ur, _cut, _chosen) in enumerate(cases):
        x[r, g.choice(vocab, m, replace=False)] = 4.0
        params[r] = (t, p, m, 0)
        u[r] = ur
    return x, params, u


@pytest.mark.parametrize("vocab", [4096, 49152])
@pytest.mark.parametrize("cap", [64, 1024])
def test_finalize_replays_at_exact_boundaries(torch_cuda, oracle, vocab, cap):  # noqa: F811
    cases = [c for c in BOUNDARY_CASES if c[0] <= cap]
    x, params, u = boundary_rows(vocab, cases, seed=vocab + cap)
    got = run_gpu(torch_cuda, x, params, u, cap)
    assert_parity(oracle, x, params, u, cap, got)
    out, ids, _ = got
    for r, (m, _t, _p, _u, cut, chosen) in enumerate(cases):
        assert int(out[r]["considered_count"]) == cut, f"row {r}"
        maxima = np.sort(np.nonzero(x[r] == 4.0)[0])
        assert int(out[r]["id"]) == int(maxima[chosen]), f"row {r}"
        assert int(out[r]["reserved"]) == 1, f"row {r}: the sequential replay did not decide"
