"""Host topology: the NUMA node closest to a GPU.

Behaviour of the reference (lmcache_ascend/v1/system_detection.py:21-45):
the GPU's PCI bus id gives ``/sys/bus/pci/devices/<bus id>/numa_node``;
some machines report -1 there (no affinity information), which is treated
as "unknown" rather than passed on to the NUMA allocator.
"""

from __future__ import annotations

import os
from typing import Callable, Dict, Optional

from .logging import init_logger

logger = init_logger(__name__)

SYSFS_PCI = "/sys/bus/pci/devices"


def _bus_id(device_index: int) -> str:
    from .. import ops

    return ops.native().get_gpu_pci_bus_id(device_index)


def numa_node_of_gpu(device_index: int, bus_id_fn: Optional[Callable[[int], str]] = None,
                     sysfs: str = SYSFS_PCI) -> Optional[int]:
    """NUMA node of GPU ``device_index``, or None when unknown (-1, missing)."""
    try:
        bus = (bus_id_fn or _bus_id)(device_index).lower()
        with open(os.path.join(sysfs, bus, "numa_node")) as f:
            node = int(f.read().strip())
    except Exception as e:  # no sysfs entry, no driver, no extension
        logger.warning("NUMA node of GPU %d unknown: %s", device_index, e)
        return None
    if node < 0:
        logger.warning("GPU %d reports NUMA node %d: no affinity, not binding", device_index,
                       node)
        return None
    return node


def gpu_to_numa_mapping(num_devices: int, **kw) -> Dict[int, int]:
    out = {}
    for i in range(num_devices):
        n = numa_node_of_gpu(i, **kw)
        if n is not None:
            out[i] = n
    return out


def resolve_numa_node(config_value: int, device_index: Optional[int]) -> int:
    """Config ``numa_node``: >= 0 binds to that node, -1 disables binding,
    -2 ("auto") binds to the GPU's node when the host reports one."""
    if config_value != -2:
        return config_value
    if device_index is None:
        return -1
    n = numa_node_of_gpu(device_index)
    return -1 if n is None else n
