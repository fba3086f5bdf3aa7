"""Host-side NUMA placement used by the host-buffer pipeline: the sysfs
cpulist parser and node lookup run on CPU; binding to a GPU's node and the
pinned-copy measurement need a GPU."""
import os

import pytest
import torch

from triton_ssm_b200 import host


def test_parse_cpulist():
    assert host.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert host.parse_cpulist("5") == {5}
    assert host.parse_cpulist("") == set()


def test_node_cpus_unknown_node_is_empty():
    assert host.node_cpus(10 ** 6) == set()


def test_node_cpus_match_the_allowed_set_on_single_node_hosts():
    cpus = host.node_cpus(0)
    if not cpus:
        pytest.skip("no NUMA information in sysfs")
    assert cpus & set(os.sched_getaffinity(0))


@pytest.mark.gpu
def test_bind_and_pinned_copy_rates():
    before = set(os.sched_getaffinity(0))
    try:
        info = host.bind_host_to_gpu("cuda:0")
        if info is not None:
            assert set(os.sched_getaffinity(0)) <= host.node_cpus(info["numa_node"])
        h2d, d2h = host.pinned_copy_gbs("cuda:0", nbytes=32 << 20, reps=2)
        assert h2d > 1.0 and d2h > 1.0
    finally:
        os.sched_setaffinity(0, before)
    assert torch.cuda.is_available()
