"""GPU: one process samples on two devices in turn. The row kernel's shared-memory
attribute and occupancy are set up once per device; a second device must not reuse the
first one's set-up. Skipped with fewer than two GPUs."""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu


def test_two_devices_in_one_process(oracle):
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import OUTCOME_DTYPE

    rows, cap = 64, 1024
    x, p, u = synth.config("c4", seed=5, rows=rows)
    ref, _, _ = oracle.sample_rows(x, p, u, cap)
    for dev in (0, 1, 0):
        d = torch.device("cuda", dev)
        with torch.cuda.device(d):
            s = Sampler(dev, max_top_k=cap, max_rows=rows, max_vocab=x.shape[1])
            logits = torch.from_numpy(x).to(d)
            pd = torch.from_numpy(p.view(np.uint8).copy()).to(d)
            ud = torch.from_numpy(u).to(d)
            out = torch.zeros(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=d)
            s.sample_rows_async(logits, pd, ud, out)
            torch.cuda.synchronize(d)
            o = out.cpu().numpy().view(OUTCOME_DTYPE)
            assert (o["status"] == 0).all()
            np.testing.assert_array_equal(o["id"], ref["id"])
            s.close()
