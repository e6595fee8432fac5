"""NUMA node of a GPU from sysfs, with the -1 sanitise (fake sysfs, CPU)."""

from lmcache_ascend_b200.utils.system_detection import (gpu_to_numa_mapping, numa_node_of_gpu,
                                                        resolve_numa_node)


def _sysfs(tmp_path, entries):
    for bus, node in entries.items():
        d = tmp_path / bus
        d.mkdir()
        (d / "numa_node").write_text(f"{node}\n")
    return str(tmp_path)


def test_numa_node_read_and_sanitised(tmp_path):
    root = _sysfs(tmp_path, {"0000:1b:00.0": 1, "0000:43:00.0": -1})
    bus = {0: "0000:1B:00.0", 1: "0000:43:00.0", 2: "0000:99:00.0"}.__getitem__
    assert numa_node_of_gpu(0, bus_id_fn=bus, sysfs=root) == 1  # bus id case-folded
    assert numa_node_of_gpu(1, bus_id_fn=bus, sysfs=root) is None  # -1: no affinity
    assert numa_node_of_gpu(2, bus_id_fn=bus, sysfs=root) is None  # missing entry
    assert gpu_to_numa_mapping(3, bus_id_fn=bus, sysfs=root) == {0: 1}


def test_resolve_config_values():
    assert resolve_numa_node(3, 0) == 3
    assert resolve_numa_node(-1, 0) == -1
    assert resolve_numa_node(-2, None) == -1
