"""IPC handles for KV-cache tensors shared with the cache server.

Counterpart of the reference's ``AscendIPCWrapper``
(lmcache_ascend/v1/multiprocess/custom_types.py:11-113): a tensor is
described by its storage's IPC handle plus dtype / shape / stride / storage
offset, and the device by a UUID that the receiving process maps to its own
device ordinal (ordinals differ between processes under
CUDA_VISIBLE_DEVICES).  CUDA tensors travel as CUDA IPC handles (the server
maps the worker's allocation; no copy); CPU tensors must live in shared
memory and travel as shared-memory names.  Handles are plain msgpack-able
values.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

_DTYPES = {str(d): d for d in (torch.float16, torch.bfloat16, torch.float32, torch.float64,
                               torch.int8, torch.uint8, torch.int16, torch.int32, torch.int64)}
_DTYPES.update({"torch.float8_e4m3fn": getattr(torch, "float8_e4m3fn", torch.uint8)})

_uuid_lock = threading.Lock()
_uuid_to_index: Dict[str, int] = {}


def device_uuid(index: int) -> str:
    return str(torch.cuda.get_device_properties(index).uuid)


def device_index_from_uuid(uuid: str) -> int:
    with _uuid_lock:
        if not _uuid_to_index:
            for i in range(torch.cuda.device_count()):
                _uuid_to_index[device_uuid(i)] = i
        idx = _uuid_to_index.get(uuid)
    if idx is None:
        raise RuntimeError(f"device {uuid} is not visible to this process")
    return idx


@dataclass
class IPCTensorHandle:
    kind: str                 # "cuda" or "cpu"
    handle: List[Any]
    dtype: str
    shape: Tuple[int, ...]
    stride: Tuple[int, ...]
    storage_offset: int
    device_uuid: str = ""

    @classmethod
    def from_tensor(cls, t: torch.Tensor) -> "IPCTensorHandle":
        st = t.untyped_storage()
        if t.is_cuda:
            h = list(st._share_cuda_())
            return cls("cuda", h, str(t.dtype), tuple(t.shape), tuple(t.stride()),
                       int(t.storage_offset()), device_uuid(t.device.index))
        if not st.is_shared():
            raise ValueError("CPU KV caches must live in shared memory (tensor.share_memory_())")
        h = list(st._share_filename_cpu_())
        return cls("cpu", h, str(t.dtype), tuple(t.shape), tuple(t.stride()),
                   int(t.storage_offset()))

    def to_tensor(self) -> torch.Tensor:
        dtype = _DTYPES[self.dtype]
        if self.kind == "cuda":
            dev = device_index_from_uuid(self.device_uuid)
            st = torch.UntypedStorage._new_shared_cuda(dev, *self.handle[1:])
            t = torch.empty((), dtype=dtype, device=f"cuda:{dev}")
        else:
            st = torch.UntypedStorage._new_shared_filename_cpu(*self.handle)
            t = torch.empty((), dtype=dtype)
        t.set_(st, self.storage_offset, self.shape, self.stride)
        return t

    def to_wire(self) -> list:
        return [self.kind, self.handle, self.dtype, list(self.shape), list(self.stride),
                self.storage_offset, self.device_uuid]

    @classmethod
    def from_wire(cls, w: Sequence) -> "IPCTensorHandle":
        h = list(w[1])
        if w[0] == "cpu":
            h = [x.encode() if isinstance(x, str) else x for x in h]
        return cls(w[0], h, w[2], tuple(w[3]), tuple(w[4]), int(w[5]), w[6])


def wrap_kv_caches(kv_caches) -> list:
    """Per-layer caches (tensor or tuple of planes) -> wire form."""
    out = []
    for layer in kv_caches:
        planes = layer if isinstance(layer, (tuple, list)) else (layer,)
        out.append([isinstance(layer, (tuple, list)),
                    [IPCTensorHandle.from_tensor(p).to_wire() for p in planes]])
    return out


def unwrap_kv_caches(wire) -> list:
    out = []
    for is_tuple, planes in wire:
        ts = [IPCTensorHandle.from_wire(p).to_tensor() for p in planes]
        out.append(tuple(ts) if is_tuple else ts[0])
    return out
