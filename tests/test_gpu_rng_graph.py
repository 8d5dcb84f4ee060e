"""Device-side draws and CUDA-graph replay of the decode step.

tabby_sample_rows_rng_async keeps each row's SeededRandom state (sampler.ts:105-119) on
the device and advances it exactly where sampleFromTopK calls random.next()
(sampler.ts:194): rows with temperature > 0 only (greedy rows return first,
sampler.ts:159-167). The reference: the same rows through tabby_sample_rows_async with
uniforms drawn on the host by SeededRandom under the same rule, step after step. Bar:
identical outcomes (ids, counts, probabilities) and identical final states.

The call depends on no host state that changes between calls (the launch epoch lives in
the device scratch), so one captured CUDA graph replays the step; replays are checked
against uncaptured calls on the same inputs.
"""
import numpy as np
import pytest

from tests.conftest import gpu_available

pytestmark = pytest.mark.gpu

VOCAB = 32768


@pytest.fixture(scope="module")
def torch_cuda():
    if not gpu_available():
        pytest.skip("no CUDA device")
    import torch

    return torch


def make_batch(rows, step, seed=0):
    from tabby_b200.sampler import PARAMS_DTYPE

    g = np.random.default_rng(seed * 1000 + step)
    x = (3.0 * g.standard_normal((rows, VOCAB))).astype(np.float32)
    p = np.zeros(rows, PARAMS_DTYPE)
    p["temperature"] = np.where(np.arange(rows) % 4 == 0, 0.0, g.uniform(0.3, 1.5, rows))
    p["top_k"] = g.choice(np.array([0, 1, 20, 64, 300]), rows)
    p["top_p"] = g.uniform(0.5, 1.0, rows)
    return x, p


def host_uniforms(states, p):
    """One SeededRandom.next() for every row that samples (temperature > 0)."""
    from tabby_b200.sampler import SeededRandom

    u = np.zeros(len(states), np.float64)
    for r, st in enumerate(states):
        if p["temperature"][r] > 0:
            g = SeededRandom(0)
            g._state = int(st)
            u[r] = g.next()
            states[r] = g._state
    return u


def run_host_u(torch, s, x, p, u):
    from tabby_b200._lib import OUTCOME_DTYPE

    dev = torch.device("cuda", 0)
    out = torch.empty(len(p) * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    s.sample_rows_async(torch.from_numpy(x).to(dev), torch.from_numpy(p.view(np.uint8)).to(dev),
                        torch.from_numpy(u).to(dev), out)
    return out.cpu().numpy().view(OUTCOME_DTYPE)


@pytest.mark.parametrize("rows", [8, 300])  # chunked rows / whole rows a CTA
def test_device_rng_matches_host_draws(torch_cuda, rows):
    torch = torch_cuda
    from tabby_b200 import Sampler
    from tabby_b200._lib import OUTCOME_DTYPE

    dev = torch.device("cuda", 0)
    s = Sampler(0, max_top_k=1024, max_rows=rows, max_vocab=VOCAB)
    seeds = (np.arange(rows, dtype=np.uint64) * 2654435761 + 12345) & 0xFFFFFFFF
    host_states = [int(v) for v in seeds]
    state_dev = torch.from_numpy(seeds.astype(np.uint32).view(np.int32)).to(dev)
    out = torch.empty(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    for step in range(3):
        x, p = make_batch(rows, step)
        s.sample_rows_rng_async(torch.from_numpy(x).to(dev),
                                torch.from_numpy(p.view(np.uint8)).to(dev), state_dev, out)
        got = out.cpu().numpy().view(OUTCOME_DTYPE).copy()
        want = run_host_u(torch, s, x, p, host_uniforms(host_states, p))
        assert (got["status"] == 0).all()
        np.testing.assert_array_equal(got["id"], want["id"])
        np.testing.assert_array_equal(got["considered_count"], want["considered_count"])
        np.testing.assert_array_equal(got["probability"], want["probability"])
        np.testing.assert_array_equal(got["pool_exhausted"], want["pool_exhausted"])
        dev_states = state_dev.cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(dev_states, np.array(host_states, np.uint32))
    s.close()


@pytest.mark.parametrize("rows", [8, 300])
def test_captured_step_replays(torch_cuda, rows):
    torch = torch_cuda
    from tabby_b200 import Sampler
    from tabby_b200._lib import OUTCOME_DTYPE

    dev = torch.device("cuda", 0)
    s = Sampler(0, max_top_k=1024, max_rows=rows, max_vocab=VOCAB)
    x0, p = make_batch(rows, 0, seed=1)
    seeds = (np.arange(rows, dtype=np.uint64) * 40503 + 7) & 0xFFFFFFFF
    logits = torch.from_numpy(x0).to(dev)
    params = torch.from_numpy(p.view(np.uint8)).to(dev)
    state = torch.from_numpy(seeds.astype(np.uint32).view(np.int32)).to(dev)
    out = torch.empty(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ref_state = state.clone()
    ref_out = torch.empty_like(out)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # warm-up outside the capture (one-time setup)
        s.sample_rows_rng_async(logits, params, state.clone(), out)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        s.sample_rows_rng_async(logits, params, state, out)
    torch.cuda.synchronize(dev)
    # Capture runs nothing: the state is still the seeds.
    np.testing.assert_array_equal(state.cpu().numpy().view(np.uint32), seeds.astype(np.uint32))

    for step in range(4):
        x, _ = make_batch(rows, step + 1, seed=1)
        logits.copy_(torch.from_numpy(x).to(dev))
        graph.replay()
        s.sample_rows_rng_async(logits, params, ref_state, ref_out)
        torch.cuda.synchronize(dev)
        got = out.cpu().numpy().view(OUTCOME_DTYPE)
        want = ref_out.cpu().numpy().view(OUTCOME_DTYPE)
        assert (got["status"] == 0).all()
        np.testing.assert_array_equal(got["id"], want["id"])
        np.testing.assert_array_equal(got["considered_count"], want["considered_count"])
        np.testing.assert_array_equal(got["probability"], want["probability"])
        np.testing.assert_array_equal(state.cpu().numpy(), ref_state.cpu().numpy())
    del graph
    s.close()


def test_drop_in_sample_batch_agrees_with_device_states(torch_cuda):
    """The host drop-in (Sampler.sample_batch with one SeededRandom a row, greedy steps
    included) and the device-RNG path agree draw for draw: same ids every step and the
    same generator states at the end (greedy steps leave both untouched)."""
    torch = torch_cuda
    from tabby_b200 import Sampler
    from tabby_b200._lib import OUTCOME_DTYPE
    from tabby_b200.sampler import SamplingParams, SeededRandom

    rows = 6
    dev = torch.device("cuda", 0)
    s = Sampler(0, max_top_k=1024, max_rows=rows, max_vocab=VOCAB)
    seeds = [11 + 977 * r for r in range(rows)]
    gens = [SeededRandom(sd) for sd in seeds]
    state_dev = torch.from_numpy(np.array(seeds, np.uint32).view(np.int32)).to(dev)
    out = torch.empty(rows * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    for step in range(5):
        x, p = make_batch(rows, step, seed=3)
        p["temperature"][(np.arange(rows) + step) % 3 == 0] = 0.0  # greedy rows move around
        xd = torch.from_numpy(x).to(dev)
        s.sample_rows_rng_async(xd, torch.from_numpy(p.view(np.uint8)).to(dev), state_dev, out)
        got = out.cpu().numpy().view(OUTCOME_DTYPE).copy()
        for r in range(rows):
            prm = SamplingParams(temperature=float(p["temperature"][r]),
                                 topK=int(p["top_k"][r]), topP=float(p["top_p"][r]))
            host = s.sample_batch(xd[r:r + 1], prm, gens[r])
            assert int(host.ids[0]) == int(got["id"][r]), (step, r)
    np.testing.assert_array_equal(state_dev.cpu().numpy().view(np.uint32),
                                  np.array([g._state for g in gens], np.uint32))
    s.close()
