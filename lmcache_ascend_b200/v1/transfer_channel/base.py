"""Transfer-channel interface: registered buffers addressed as (uuid, page).

A channel owns a set of local buffers split into fixed-size pages and maps
the peers' buffers after a handshake.  Remote memory is always named as
``(buffer_uuid, page_index)`` and never as a raw pointer, as in the
reference (lmcache_ascend/v1/transfer_channel/hccl_channel.py:559-590,
buffer_config.py:85-93).  Concrete channels: ``NVLinkChannel`` (CUDA IPC +
peer copies on one box) and ``TCPChannel`` (host buffers over ZMQ; CPU tier
and cross-box fallback).
"""

from __future__ import annotations

import abc
import threading
import uuid as _uuid
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

RemoteAddr = Tuple[str, int]  # (buffer uuid, page index)


@dataclass
class BufferConfig:
    tensor: torch.Tensor          # uint8 [nbytes], device or host
    page_bytes: int
    uuid: str = field(default_factory=lambda: _uuid.uuid4().hex)
    shm_name: Optional[str] = None  # host buffers shared by name across processes

    @property
    def kind(self) -> str:
        if self.tensor.is_cuda:
            return "device"
        return "host_shm" if self.shm_name else "host"

    @property
    def nbytes(self) -> int:
        return self.tensor.numel()

    def page_ptr(self, index: int) -> int:
        return self.tensor.data_ptr() + index * self.page_bytes


@dataclass
class RemoteBuffer:
    uuid: str
    kind: str
    nbytes: int
    page_bytes: int
    va: int = 0                       # mapped address (NVLink channel)
    tensor: Optional[torch.Tensor] = None  # attached host view (shm)


class BaseTransferChannel(abc.ABC):
    def __init__(self, peer_id: str, buffers: Optional[Sequence[BufferConfig]] = None):
        self.peer_id = peer_id
        self.local: Dict[str, BufferConfig] = {}
        self.remote: Dict[str, Dict[str, RemoteBuffer]] = {}  # peer -> uuid -> buffer
        self._lock = threading.RLock()
        for b in buffers or []:
            self.register_buffer(b)

    # ------------------------------------------------------------ buffers
    def register_buffer(self, buf: BufferConfig) -> str:
        with self._lock:
            self.local[buf.uuid] = buf
        return buf.uuid

    def get_local_buffer_refs(self) -> List[dict]:
        return [self._export(b) for b in self.local.values()]

    @abc.abstractmethod
    def _export(self, buf: BufferConfig) -> dict: ...

    @abc.abstractmethod
    def lazy_init_peer_connection(self, peer_id: str, refs: List[dict],
                                  endpoint: Optional[str] = None) -> None: ...

    def remote_xfer_handler_exists(self, peer_id: str) -> bool:
        return peer_id in self.remote

    def resolve(self, peer_id: str, addr: RemoteAddr) -> RemoteBuffer:
        try:
            return self.remote[peer_id][addr[0]]
        except KeyError:
            raise KeyError(f"unknown remote buffer {addr[0]} of peer {peer_id}")

    # ---------------------------------------------------------- transfers
    @abc.abstractmethod
    def batched_write(self, srcs: Sequence[Tuple[int, int]], peer_id: str,
                      remote: Sequence[RemoteAddr], sync: bool = True): ...

    @abc.abstractmethod
    def batched_read(self, dsts: Sequence[Tuple[int, int]], peer_id: str,
                     remote: Sequence[RemoteAddr], sync: bool = True): ...

    def submit_batched_read(self, dsts, peer_id, remote):
        """Asynchronous read: returns an object with ``synchronize()``/``query()``."""
        return self.batched_read(dsts, peer_id, remote, sync=False)

    def close(self) -> None:
        pass


class CompletedEvent:
    """Stand-in for a CUDA event of a transfer that already completed."""

    def synchronize(self) -> None:
        return None

    def query(self) -> bool:
        return True
