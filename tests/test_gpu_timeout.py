"""GPU: a bounded device wait that runs out is reported, not hidden.

The row pass waits (bounded) for each row's plan entry before streaming the row's units.
The test-only entry tabby_sample_rows_debug_async never publishes one row's plan and
limits the wait to a few thousand polls. The kernel must return; that row must report
TABBY_ETIMEOUT; every other row must equal the oracle exactly; and the next ordinary call
on the same handle must be correct. The reference reports device failure as an error
(src/worker/inference.worker.ts:55-58, onDeviceLost -> fail). No GPU fault is involved:
the wait simply gives up.
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu

REL = 1e-5


def _device_arrays(torch, x, p, u):
    from tabby_b200._lib import OUTCOME_DTYPE

    rows = x.shape[0]
    logits = torch.from_numpy(x).cuda()
    pd = torch.from_numpy(p.view(np.uint8).copy()).cuda()
    ud = torch.from_numpy(u).cuda()
    out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device="cuda")
    return logits, pd, ud, out


def _check_row(o, e):
    assert o["status"] == 0
    assert int(o["id"]) == int(e["id"])
    assert int(o["considered_count"]) == int(e["considered_count"])
    assert int(o["pool_size"]) == int(e["pool_size"])
    assert np.float32(o["max_logit"]) == np.float32(e["max_logit"])
    assert abs(float(o["sum_exp"]) - float(e["sum_exp"])) <= REL * float(e["sum_exp"])
    assert abs(o["probability"] - e["probability"]) <= REL * e["probability"]


@pytest.mark.parametrize("withheld", [0, 5])
def test_withheld_plan_reports_timeout_and_the_rest_is_exact(oracle, withheld):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import OUTCOME_DTYPE, TABBY_ETIMEOUT, check, lib

    L = lib()
    rows, cap = 8, 1024
    x, p, u = synth.config("c4", seed=77, rows=rows)
    p["top_k"] = np.array([0, 20, 100, 1000, 1, 40, 7, 200])
    ref, _, _ = oracle.sample_rows(x, p, u, cap)
    s = Sampler(0, max_top_k=cap, max_rows=rows, max_vocab=x.shape[1])
    logits, pd, ud, out = _device_arrays(torch, x, p, u)
    stream = torch.cuda.current_stream().cuda_stream
    check(L.tabby_sample_rows_debug_async(s.handle, logits.data_ptr(), x.shape[1], rows,
                                          x.shape[1], pd.data_ptr(), ud.data_ptr(),
                                          out.data_ptr(), 2000, withheld, stream))
    torch.cuda.synchronize()
    o = out.cpu().numpy().view(OUTCOME_DTYPE)
    assert int(o[withheld]["status"]) == TABBY_ETIMEOUT
    assert int(o[withheld]["id"]) == -1
    for r in range(rows):
        if r != withheld:
            _check_row(o[r], ref[r])
    # The handle stays usable: the next ordinary call is exact on every row.
    out.zero_()
    s.sample_rows_async(logits, pd, ud, out)
    torch.cuda.synchronize()
    o = out.cpu().numpy().view(OUTCOME_DTYPE)
    for r in range(rows):
        _check_row(o[r], ref[r])
    s.close()


def test_debug_entry_without_withholding_equals_the_normal_entry(oracle):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import OUTCOME_DTYPE, check, lib

    L = lib()
    rows, cap = 16, 1024
    x, p, u = synth.config("c4", seed=78, rows=rows)
    ref, _, _ = oracle.sample_rows(x, p, u, cap)
    s = Sampler(0, max_top_k=cap, max_rows=rows, max_vocab=x.shape[1])
    logits, pd, ud, out = _device_arrays(torch, x, p, u)
    check(L.tabby_sample_rows_debug_async(s.handle, logits.data_ptr(), x.shape[1], rows,
                                          x.shape[1], pd.data_ptr(), ud.data_ptr(),
                                          out.data_ptr(), 1 << 24, -1,
                                          torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    o = out.cpu().numpy().view(OUTCOME_DTYPE)
    for r in range(rows):
        _check_row(o[r], ref[r])
    s.close()
