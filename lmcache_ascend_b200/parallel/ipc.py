"""CUDA IPC descriptors for device memory shared between processes.

A descriptor names a device address as (IPC handle of its allocation, byte
offset, device, owner pid) so it can travel through any control channel
(torch.distributed object collectives, ZMQ, a TCP store).  The reference
ships HCCL/HIXL RMA descriptors the same way (reference
lmcache_ascend/v1/transfer_channel/hccl_channel.py:140-280) and never raw
pointers across processes.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .. import ops


@dataclass(frozen=True)
class IpcDesc:
    handle: bytes
    offset: int
    alloc_size: int
    device: int
    pid: int
    pci_bus_id: str = ""

    def to_dict(self) -> dict:
        return {"handle": self.handle, "offset": self.offset, "alloc_size": self.alloc_size,
                "device": self.device, "pid": self.pid, "pci_bus_id": self.pci_bus_id}

    @staticmethod
    def from_dict(d: dict) -> "IpcDesc":
        return IpcDesc(d["handle"], d["offset"], d["alloc_size"], d["device"], d["pid"],
                       d.get("pci_bus_id", ""))


def export_ptr(ptr: int, device: int) -> IpcDesc:
    handle, offset, size = ops.native().ipc_export(int(ptr), int(device))
    try:
        bus = ops.native().get_gpu_pci_bus_id(int(device))
    except Exception:  # pragma: no cover
        bus = ""
    return IpcDesc(bytes(handle), int(offset), int(size), int(device), os.getpid(), bus)


def export_tensor(t: torch.Tensor) -> IpcDesc:
    if not t.is_cuda:
        raise ValueError("only device tensors can be exported over CUDA IPC")
    return export_ptr(t.data_ptr(), t.device.index or 0)


class PeerMappings:
    """Opened peer allocations of this process (ref counted per handle)."""

    def __init__(self, device: int):
        self.device = int(device)
        self._opened: Dict[bytes, int] = {}

    def resolve(self, desc: IpcDesc) -> int:
        """Device VA (in this process) of the described address."""
        if desc.pid == os.getpid():
            # same process (loopback): the exporter's VA is valid here; CUDA
            # refuses to open an IPC handle in the process that exported it
            return self._local_va(desc)
        va = int(ops.native().ipc_import(desc.handle, desc.offset, self.device))
        self._opened[desc.handle] = self._opened.get(desc.handle, 0) + 1
        return va

    _local: Dict[bytes, int] = {}

    @classmethod
    def register_local(cls, desc: IpcDesc, ptr: int) -> None:
        cls._local[(desc.handle, desc.offset)] = ptr

    def _local_va(self, desc: IpcDesc) -> int:
        key = (desc.handle, desc.offset)
        if key not in self._local:
            raise KeyError("local IPC descriptor was not registered in this process")
        return self._local[key]

    def close(self) -> None:
        mod = ops.native()
        for h, n in self._opened.items():
            for _ in range(n):
                mod.ipc_close(h)
        self._opened.clear()


def export_local(ptr: int, device: int) -> IpcDesc:
    """Export and remember the local VA so a same-process peer resolves it."""
    d = export_ptr(ptr, device)
    PeerMappings.register_local(d, int(ptr))
    return d
