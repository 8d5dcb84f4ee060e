"""Host-side helpers of bench.py that need no GPU: the sysfs cpulist parser and the
NUMA-local block the end-to-end leg allocates its pinned buffers in."""
import os

import bench


def test_parse_cpulist():
    assert bench.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert bench.parse_cpulist("5") == {5}
    assert bench.parse_cpulist("") == set()


def test_numa_local_restores_affinity(monkeypatch):
    before = os.sched_getaffinity(0)
    one = {min(before)}
    monkeypatch.setattr(bench, "gpu_numa_cpus", lambda dev: (0, one))
    with bench.NumaLocal(0) as numa:
        assert numa.node == 0
        assert os.sched_getaffinity(0) == one
    assert os.sched_getaffinity(0) == before


def test_numa_local_without_node_is_a_no_op(monkeypatch):
    before = os.sched_getaffinity(0)
    monkeypatch.setattr(bench, "gpu_numa_cpus", lambda dev: (None, None))
    with bench.NumaLocal(0) as numa:
        assert numa.node is None
        assert os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before
