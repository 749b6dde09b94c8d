"""Host-side helpers of the pipeline: the cpulist parser and the NUMA binding,
which must change nothing where the GPU's node cannot be read."""
import os

from fast_forced_aligner_b200.pipeline import bind_host_to_device, parse_cpulist


def test_parse_cpulist():
    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert parse_cpulist("5") == [5]
    assert parse_cpulist("") == []


def test_binding_without_a_readable_node_changes_nothing():
    before = os.sched_getaffinity(0)
    cpus = bind_host_to_device(0)
    if cpus is None:
        assert os.sched_getaffinity(0) == before
    else:  # a GPU host: the process now runs on that node's CPUs
        assert set(cpus) == os.sched_getaffinity(0)
        os.sched_setaffinity(0, before)
