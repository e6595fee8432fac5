"""Memory objects and allocators (chunk storage).

Re-creates the upstream LMCache memory layer the reference builds on
(``MemoryObj``, ``MemoryFormat``, pinned / paged allocators; patched by
reference lmcache_ascend/v1/memory_management.py:20-54): a chunk is a
``MemoryObj`` -- a typed tensor view into a large registered buffer with a
reference count (owners) and a pin count (in-flight lookups/transfers).

B200 specifics: host buffers are ``cudaHostAlloc(Mapped|Portable)`` pinned
memory from the native allocator (so the copy engines reach full PCIe rate
and kernels may read them zero-copy), optionally NUMA-bound or POSIX-shm
backed; device buffers come from ``cudaMalloc`` so they can be exported to a
peer GPU over CUDA IPC.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable, List, Optional, Tuple

import torch
from sortedcontainers import SortedDict

from ..utils.logging import init_logger

logger = init_logger(__name__)

ALIGN = 256


class MemoryFormat(Enum):
    UNDEFINED = 0
    KV_2LTD = 1     # [2, L, T, H*D]
    KV_T2D = 2      # [T, 2, H*D] (one layer, token-major)
    KV_MLA_FMT = 3  # [1, L, T, D_total]
    BINARY = 4      # serialized bytes (remote / cachegen)
    BINARY_BUFFER = 5

    def token_dim(self) -> int:
        return {MemoryFormat.KV_2LTD: 2, MemoryFormat.KV_T2D: 0,
                MemoryFormat.KV_MLA_FMT: 2}.get(self, -1)


def _dtype_size(dtype: torch.dtype) -> int:
    return dtype.itemsize


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


@dataclass
class MemoryObjMetadata:
    shape: torch.Size
    dtype: Optional[torch.dtype]
    address: int          # byte offset inside the allocator's buffer
    phy_size: int         # bytes reserved
    fmt: MemoryFormat = MemoryFormat.UNDEFINED
    ref_count: int = 1
    pin_count: int = 0
    cached_positions: Optional[torch.Tensor] = None


class MemoryObj:
    """A chunk of KV data owned by an allocator.

    ``ref_count`` counts owners (storage backends, in-flight transfers);
    reaching zero returns the memory.  ``pin_count`` protects objects that a
    lookup promised to a later retrieve from eviction.
    """

    def __init__(self, raw: Optional[torch.Tensor], meta: MemoryObjMetadata,
                 allocator: Optional["BaseAllocator"] = None):
        self.raw_data = raw  # uint8 view of the reserved bytes
        self.meta = meta
        self._allocator = allocator
        self._lock = threading.Lock()
        self._valid = True

    # ---- views
    @property
    def tensor(self) -> Optional[torch.Tensor]:
        if self.raw_data is None or self.meta.dtype is None:
            return None
        nbytes = _numel(self.meta.shape) * _dtype_size(self.meta.dtype)
        return self.raw_data[:nbytes].view(self.meta.dtype).view(self.meta.shape)

    @property
    def byte_array(self) -> bytes:
        t = self.raw_data
        n = self.get_size()
        return bytes(t[:n].cpu().numpy().tobytes())

    @property
    def metadata(self) -> MemoryObjMetadata:
        return self.meta

    def get_shape(self) -> torch.Size:
        return self.meta.shape

    def get_dtype(self) -> Optional[torch.dtype]:
        return self.meta.dtype

    def get_memory_format(self) -> MemoryFormat:
        return self.meta.fmt

    def get_size(self) -> int:
        if self.meta.dtype is None:
            return _numel(self.meta.shape)
        return _numel(self.meta.shape) * _dtype_size(self.meta.dtype)

    def get_physical_size(self) -> int:
        return self.meta.phy_size

    def get_num_tokens(self) -> int:
        d = self.meta.fmt.token_dim()
        return int(self.meta.shape[d]) if d >= 0 else 0

    def data_ptr(self) -> int:
        return self.raw_data.data_ptr() if self.raw_data is not None else 0

    @property
    def is_valid(self) -> bool:
        return self._valid

    # ---- reference counting
    def ref_count_up(self, n: int = 1) -> None:
        with self._lock:
            self.meta.ref_count += n

    def ref_count_down(self, n: int = 1) -> None:
        free = False
        with self._lock:
            self.meta.ref_count -= n
            if self.meta.ref_count < 0:
                logger.error("negative ref count on %s", self.meta)
                self.meta.ref_count = 0
            free = self.meta.ref_count == 0 and self._valid
        if free:
            self.free()

    def get_ref_count(self) -> int:
        return self.meta.ref_count

    def pin(self) -> bool:
        with self._lock:
            self.meta.pin_count += 1
        return True

    def unpin(self) -> bool:
        with self._lock:
            if self.meta.pin_count > 0:
                self.meta.pin_count -= 1
        return True

    @property
    def is_pinned(self) -> bool:
        return self.meta.pin_count > 0

    def free(self) -> None:
        if not self._valid:
            return
        self._valid = False
        if self._allocator is not None:
            self._allocator._release(self)

    def __repr__(self) -> str:
        return (f"MemoryObj(shape={tuple(self.meta.shape)}, dtype={self.meta.dtype}, "
                f"fmt={self.meta.fmt.name}, ref={self.meta.ref_count}, "
                f"pin={self.meta.pin_count}, addr={self.meta.address})")


class BytesMemoryObj(MemoryObj):
    """A serialized chunk held as Python bytes (remote/cachegen payloads)."""

    def __init__(self, data: bytes, fmt: MemoryFormat = MemoryFormat.BINARY):
        meta = MemoryObjMetadata(torch.Size([len(data)]), None, 0, len(data), fmt)
        super().__init__(None, meta, None)
        self._bytes = data

    @property
    def byte_array(self) -> bytes:
        return self._bytes

    def get_size(self) -> int:
        return len(self._bytes)


class BaseAllocator:
    """Interface shared by all allocators."""

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD
                 ) -> Optional[MemoryObj]:
        raise NotImplementedError

    def batched_allocate(self, shape, dtype, batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD
                         ) -> Optional[List[MemoryObj]]:
        objs = []
        for _ in range(batch_size):
            o = self.allocate(shape, dtype, fmt)
            if o is None:
                for p in objs:
                    p.ref_count_down()
                return None
            objs.append(o)
        return objs

    def _release(self, obj: MemoryObj) -> None:
        raise NotImplementedError

    def close(self) -> None:
        pass


class TensorMemoryAllocator(BaseAllocator):
    """Best-fit allocator over one byte buffer with free-block coalescing.

    Free blocks are kept in two sorted maps (by address and by size) so
    allocate/free are O(log n).
    """

    def __init__(self, buffer: torch.Tensor, align: int = ALIGN):
        assert buffer.dtype == torch.uint8 and buffer.dim() == 1
        self.buffer = buffer
        self.align = align
        self.capacity = buffer.numel()
        self._lock = threading.Lock()
        self._free_by_addr = SortedDict({0: self.capacity})
        self._free_by_size = SortedDict({(self.capacity, 0): None})
        self.used_bytes = 0
        self.num_active = 0

    def _round(self, n: int) -> int:
        return (n + self.align - 1) // self.align * self.align

    def _take(self, size: int) -> Optional[int]:
        i = self._free_by_size.bisect_left((size, -1))
        if i >= len(self._free_by_size):
            return None
        (bsize, addr), _ = self._free_by_size.peekitem(i)
        del self._free_by_size[(bsize, addr)]
        del self._free_by_addr[addr]
        if bsize > size:
            self._free_by_addr[addr + size] = bsize - size
            self._free_by_size[(bsize - size, addr + size)] = None
        return addr

    def _give(self, addr: int, size: int) -> None:
        # coalesce with successor
        nxt = self._free_by_addr.get(addr + size)
        if nxt is not None:
            del self._free_by_addr[addr + size]
            del self._free_by_size[(nxt, addr + size)]
            size += nxt
        # coalesce with predecessor
        i = self._free_by_addr.bisect_left(addr)
        if i > 0:
            paddr, psize = self._free_by_addr.peekitem(i - 1)
            if paddr + psize == addr:
                del self._free_by_addr[paddr]
                del self._free_by_size[(psize, paddr)]
                addr, size = paddr, psize + size
        self._free_by_addr[addr] = size
        self._free_by_size[(size, addr)] = None

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD
                 ) -> Optional[MemoryObj]:
        shape = torch.Size(shape)
        nbytes = _numel(shape) * (_dtype_size(dtype) if dtype is not None else 1)
        size = self._round(max(nbytes, 1))
        with self._lock:
            addr = self._take(size)
            if addr is None:
                return None
            self.used_bytes += size
            self.num_active += 1
        raw = self.buffer[addr:addr + size]
        return MemoryObj(raw, MemoryObjMetadata(shape, dtype, addr, size, fmt), self)

    def _release(self, obj: MemoryObj) -> None:
        with self._lock:
            self._give(obj.meta.address, obj.meta.phy_size)
            self.used_bytes -= obj.meta.phy_size
            self.num_active -= 1

    def memcheck(self) -> bool:
        """Free + used bytes account for the whole buffer, no overlaps."""
        with self._lock:
            free = sum(self._free_by_addr.values())
            prev_end = -1
            for a, s in self._free_by_addr.items():
                if a < prev_end:
                    return False
                prev_end = a + s
            return free + self.used_bytes == self.capacity


class PagedTensorAllocator(BaseAllocator):
    """Fixed-size pages (one full chunk each), O(1) allocate/free.

    Used by the PD receiver buffer and the pinned CPU pool when all chunks
    have the same maximum size; a partial chunk still takes one page.
    Pages are addressed by index so a remote peer can name them as
    ``(buffer_uuid, page_index)`` (reference
    lmcache_ascend/v1/transfer_channel/hccl_channel.py:559-590).
    """

    def __init__(self, buffer: torch.Tensor, page_bytes: int, align: int = ALIGN):
        assert buffer.dtype == torch.uint8 and buffer.dim() == 1
        self.buffer = buffer
        self.page_bytes = (page_bytes + align - 1) // align * align
        self.num_pages = buffer.numel() // self.page_bytes
        if self.num_pages == 0:
            raise ValueError("buffer smaller than one page")
        self._free = list(range(self.num_pages - 1, -1, -1))
        self._lock = threading.Lock()

    @property
    def num_free(self) -> int:
        return len(self._free)

    def page_ptr(self, index: int) -> int:
        return self.buffer.data_ptr() + index * self.page_bytes

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD
                 ) -> Optional[MemoryObj]:
        shape = torch.Size(shape)
        nbytes = _numel(shape) * _dtype_size(dtype)
        if nbytes > self.page_bytes:
            raise ValueError(f"object of {nbytes} B exceeds page size {self.page_bytes}")
        with self._lock:
            if not self._free:
                return None
            idx = self._free.pop()
        addr = idx * self.page_bytes
        raw = self.buffer[addr:addr + self.page_bytes]
        return MemoryObj(raw, MemoryObjMetadata(shape, dtype, addr, self.page_bytes, fmt), self)

    def page_index(self, obj: MemoryObj) -> int:
        return obj.meta.address // self.page_bytes

    def _release(self, obj: MemoryObj) -> None:
        with self._lock:
            self._free.append(obj.meta.address // self.page_bytes)


# ---------------------------------------------------------------------------
# Buffers
# ---------------------------------------------------------------------------
class HostBuffer:
    """Pinned host buffer (native cudaHostAlloc / NUMA / shm) as a uint8 tensor.

    Falls back to pageable memory when no GPU is present (CPU-only tier).
    """

    def __init__(self, nbytes: int, numa_node: int = -1, shm_name: Optional[str] = None,
                 attach: bool = False, device: int = -1):
        from .. import ops

        self.nbytes = int(nbytes)
        self._ptr = None
        self._kind = None
        self.shm_name = shm_name
        use_native = ops.native_available()
        if use_native and (torch.cuda.is_available() or shm_name is not None or numa_node >= 0):
            mod = ops.native()
            if shm_name is not None:
                self._ptr = (mod.attach_shm_pinned_ptr(self.nbytes, shm_name) if attach else
                             mod.alloc_shm_pinned_ptr(self.nbytes, shm_name, numa_node))
                self._kind = "shm"
            elif numa_node >= 0:
                self._ptr = mod.alloc_pinned_numa_ptr(self.nbytes, numa_node)
                self._kind = "numa"
            else:
                self._ptr = mod.alloc_pinned_ptr(self.nbytes, device)
                self._kind = "pinned"
            self.tensor = mod.host_tensor_view(self._ptr, self.nbytes)
        else:
            self.tensor = torch.empty(self.nbytes, dtype=torch.uint8)
            self._kind = "pageable"

    @property
    def pinned(self) -> bool:
        return self._kind in ("pinned", "numa", "shm") and torch.cuda.is_available()

    def close(self, unlink: bool = False) -> None:
        if self._ptr is None:
            return
        from .. import ops

        mod = ops.native()
        self.tensor = None
        if self._kind == "shm":
            if unlink:
                mod.free_shm_pinned_ptr(self._ptr)
            else:
                mod.detach_shm_pinned_ptr(self._ptr)
        else:
            mod.free_pinned_ptr(self._ptr)
        self._ptr = None


class DeviceBuffer:
    """cudaMalloc'd device buffer (exportable over CUDA IPC) as a uint8 tensor."""

    def __init__(self, nbytes: int, device: torch.device):
        from .. import ops

        device = torch.device(device)
        if device.type == "cuda":
            self.tensor = ops.native().device_buffer(int(nbytes), device.index or 0)
        else:
            self.tensor = torch.zeros(int(nbytes), dtype=torch.uint8, device=device)
        self.nbytes = int(nbytes)


class PinnedMemoryAllocator(TensorMemoryAllocator):
    def __init__(self, nbytes: int, numa_node: int = -1, shm_name: Optional[str] = None,
                 attach: bool = False):
        self.host = HostBuffer(nbytes, numa_node=numa_node, shm_name=shm_name, attach=attach)
        super().__init__(self.host.tensor)

    def close(self) -> None:
        self.host.close()


class GPUMemoryAllocator(TensorMemoryAllocator):
    def __init__(self, nbytes: int, device: torch.device):
        self.dev = DeviceBuffer(nbytes, device)
        super().__init__(self.dev.tensor)
