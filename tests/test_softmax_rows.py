"""softmax_rows (the attention-score softmax next to the sampler): the CUDA kernel through the C ABI against the
oracle restatement of cpu.ts softmaxRows (fp32 rounding as the reference's CPU form).

Bar: masked tail exactly 0; every entry within the reference's own kernel tolerance of the
oracle (1e-4 absolute, kernels.test.ts:173); every kept entry within 1e-5 relative of the
exact (float64) softmax (the oracle's left-to-right fp32 sum drifts on long rows, the
kernel's tree sum does not); rows summing to 1 within 1e-5. The oracle itself is pinned first against a plain-Python form of
the reference's loop and the properties its test checks (kernels.test.ts:457-485).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from tests.conftest import gpu_available


def py_softmax_rows(x, n_rows, row_len, period, offset):
    """Plain-Python transcription of the reference loop, float64 throughout (a check of
    the oracle's indexing and masking, not of its rounding)."""
    import math

    out = list(map(float, x))
    for row in range(n_rows):
        valid = offset + (row % period) + 1 if period else row_len
        base = row * row_len
        m = max(out[base:base + valid])
        es = [math.exp(out[base + i] - m) for i in range(valid)]
        s = sum(es)
        for i in range(valid):
            out[base + i] = es[i] / s
        for i in range(valid, row_len):
            out[base + i] = 0.0
    return np.array(out).reshape(n_rows, row_len)


def ref_random_f32(count, seed, scale=1.0):
    """randomF32 of the reference's tests (tests/support.ts:7-24): mulberry32 draws mapped
    to (u * 2 - 1) * scale in float64, stored as float32."""
    a = seed & 0xFFFFFFFF
    out = np.zeros(count, np.float32)
    for i in range(count):
        a = (a + 0x6D2B79F5) & 0xFFFFFFFF
        t = a
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + (((t ^ (t >> 7)) * (t | 61)) & 0xFFFFFFFF)) & 0xFFFFFFFF
        u = ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296
        out[i] = (u * 2 - 1) * scale
    return out


def test_oracle_on_the_reference_fixture():
    """The reference test's own input: randomF32(3 * 5 * 5, 0x50f7, 4), 15 rows of 5,
    causal period 5 (kernels.test.ts:457-485)."""
    x = ref_random_f32(75, 0x50F7, 4)
    assert x.min() >= -4 and x.max() <= 4
    got = orc.softmax_rows(x, 15, 5, 5, 0)
    want = py_softmax_rows(x, 15, 5, 5, 0)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
    for r in range(15):
        valid = (r % 5) + 1
        assert (got[r, valid:] == 0).all()
        assert abs(float(got[r].astype(np.float64).sum()) - 1.0) < 1e-5


@pytest.mark.gpu
def test_gpu_on_the_reference_fixture():
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200._lib import check, lib

    x = ref_random_f32(75, 0x50F7, 4)
    d = torch.from_numpy(x.copy()).cuda()
    check(lib().tabby_softmax_rows_async(d.data_ptr(), 15, 5, 5, 0,
                                         torch.cuda.current_stream().cuda_stream))
    got = d.cpu().numpy().reshape(15, 5)
    want = orc.softmax_rows(x, 15, 5, 5, 0)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-4)  # kernels.test.ts expectClose
    for r in range(15):
        assert (got[r, (r % 5) + 1:] == 0).all()
        assert abs(float(got[r].astype(np.float64).sum()) - 1.0) < 1e-5


@pytest.mark.parametrize("n_heads,n_tokens,period,offset", [(3, 5, 5, 0), (2, 7, 0, 0),
                                                             (4, 9, 3, 6)])
def test_oracle_matches_reference_loop(n_heads, n_tokens, period, offset):
    g = np.random.default_rng(0x50F7)
    rows = n_heads * n_tokens
    x = (4 * g.standard_normal(rows * n_tokens)).astype(np.float32)
    got = orc.softmax_rows(x, rows, n_tokens, period, offset)
    want = py_softmax_rows(x, rows, n_tokens, period, offset)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
    for r in range(rows):  # the properties kernels.test.ts:475-484 checks
        valid = offset + (r % period) + 1 if period else n_tokens
        assert (got[r, valid:] == 0).all()
        assert abs(float(got[r].astype(np.float64).sum()) - 1.0) < 1e-5


CASES = [
    # (rows, row_len, causal_period, causal_offset): the reference test's shape, decode
    # (one query a head over a long context), prefill with a causal mask, long rows.
    (15, 5, 5, 0),
    (14, 2048, 1, 2047),
    (14 * 64, 64, 64, 0),
    (7 * 300, 300, 300, 0),
    (8, 3000, 0, 0),
    (4, 20000, 0, 0),
    (6, 9000, 3, 8000),
    (5, 8192, 0, 0),
    # Lengths that are not a multiple of 4 take the scalar kernels.
    (10, 1001, 0, 0),
    (6, 4099, 2, 4000),
    (3, 8191, 0, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,row_len,period,offset", CASES)
def test_gpu_softmax_rows_matches_oracle(rows, row_len, period, offset):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200._lib import check, lib

    g = np.random.default_rng(rows * 7 + row_len)
    x = (4 * g.standard_normal((rows, row_len))).astype(np.float32)
    d = torch.from_numpy(x).cuda()
    check(lib().tabby_softmax_rows_async(d.data_ptr(), rows, row_len, period, offset,
                                         torch.cuda.current_stream().cuda_stream))
    got = d.cpu().numpy()
    want = orc.softmax_rows(x, rows, row_len, period, offset)
    for r in range(rows):
        valid = offset + (r % period) + 1 if period else row_len
        assert (got[r, valid:] == 0).all()
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-4)
    exact = py_softmax_rows(x.reshape(-1), rows, row_len, period, offset)
    np.testing.assert_allclose(got, exact, rtol=1e-5, atol=1e-12)
    assert np.abs(got.astype(np.float64).sum(1) - 1.0).max() < 1e-5
