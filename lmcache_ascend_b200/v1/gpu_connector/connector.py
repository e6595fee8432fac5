"""Paged-memory GPU connectors.

Behaviour follows the reference connectors
(lmcache_ascend/v1/npu_connector/npu_connectors.py: ``VLLMPagedMemNPUConnectorV2``
:789-1486 with ``from_gpu``/``to_gpu``/``batched_*``/``get_shape``,
``VLLMPagedMemLayerwiseNPUConnector`` generators :1580-8090,
``VLLMBufferLayerwiseNPUConnector`` :405-786, SGLang connectors :8093-8376).

The B200 data path:
* chunk objects in device memory (PD buffers, GPU tier): ONE TMA-bulk kernel
  launch for the whole batch through a device table of chunk pointers;
* chunk objects in pinned host memory, ``copy_engine`` mode: per chunk a TMA
  gather into a device staging ring on ``store_stream`` and a
  ``cudaMemcpyAsync`` D2H on ``copy_stream`` (the gather of chunk i+1 overlaps
  the PCIe copy of chunk i; events order stage reuse).  Loads run the mirror
  pipeline (H2D on ``copy_stream``, scatter on ``load_stream``);
* ``zero_copy`` mode: one SIMT kernel reads/writes the host-mapped pinned
  chunks directly (no staging, one launch per batch);
* CPU tensors: the PyTorch oracle of ``PagedKVLayout`` (CPU test tier).
"""

from __future__ import annotations

import abc
from typing import Generator, List, Optional, Sequence, Tuple

import torch

from ...config import LMCacheEngineConfig
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ...utils.nvtx import nvtx_range
from ..kv_format import KVCacheFormat, PagedKVLayout
from ..memory_management import MemoryFormat, MemoryObj
from ..proxy_memory_obj import is_proxy, load_proxies_pipelined

logger = init_logger(__name__)

_MODE = {"auto": 0, "tma": 1, "simt": 2}


class GPUConnectorInterface(abc.ABC):
    @abc.abstractmethod
    def get_shape(self, num_tokens: int) -> torch.Size: ...

    @abc.abstractmethod
    def batched_from_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                         ends: Sequence[int], **kwargs) -> None: ...

    @abc.abstractmethod
    def batched_to_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                       ends: Sequence[int], **kwargs) -> None: ...

    def from_gpu(self, memory_obj: MemoryObj, start: int, end: int, **kwargs) -> None:
        self.batched_from_gpu([memory_obj], [start], [end], **kwargs)

    def to_gpu(self, memory_obj: MemoryObj, start: int, end: int, **kwargs) -> None:
        self.batched_to_gpu([memory_obj], [start], [end], **kwargs)


class VLLMPagedMemGPUConnector(GPUConnectorInterface):
    """Whole-chunk (all layers) transfers between vLLM's paged cache and chunks."""

    def __init__(self, config: Optional[LMCacheEngineConfig] = None, device=None,
                 use_mla: bool = False, kvcaches=None, num_stages: int = 4):
        self.config = config or LMCacheEngineConfig()
        self.use_mla = use_mla
        self.device = torch.device(device) if device is not None else None
        self.layout: Optional[PagedKVLayout] = None
        self.num_stages = num_stages
        self._stages: List[torch.Tensor] = []
        self._stage_free: List[Optional[torch.cuda.Event]] = []
        self.store_stream = None
        self.load_stream = None
        self.copy_stream = None
        self.stats = get_stats()
        if kvcaches is not None:
            self.register_kv_caches(kvcaches)

    # ------------------------------------------------------------- set-up
    def register_kv_caches(self, kvcaches, fmt: Optional[KVCacheFormat] = None) -> None:
        self.layout = PagedKVLayout(kvcaches, use_mla=self.use_mla, fmt=fmt)
        self.device = self.layout.device
        if self.device.type == "cuda":
            from ... import ops

            ops.native()  # mandatory on GPU: fail loudly if the build is missing
            self.layout.native()
            self.layout.chunk_native()
            with torch.cuda.device(self.device):
                self.store_stream = torch.cuda.Stream()
                self.load_stream = torch.cuda.Stream()
                self.copy_stream = torch.cuda.Stream()

    @property
    def kvcaches_registered(self) -> bool:
        return self.layout is not None

    def get_shape(self, num_tokens: int) -> torch.Size:
        return torch.Size(self.layout.chunk_shape(num_tokens))

    @property
    def memory_format(self) -> MemoryFormat:
        return MemoryFormat.KV_2LTD if self.layout.fmt.uses_2ltd_chunks else MemoryFormat.KV_MLA_FMT

    def chunk_bytes(self, num_tokens: int) -> int:
        return self.layout.chunk_bytes(num_tokens)

    # ------------------------------------------------------------ helpers
    def _mode(self) -> int:
        return _MODE[self.config.gpu_transfer_mode]

    def _native_xfer(self, chunk: Optional[torch.Tensor], slots: torch.Tensor,
                     to_chunk: bool, chunk_ptrs: Optional[torch.Tensor] = None,
                     chunk_tokens: int = 0, chunk_on_device: bool = True,
                     layer_begin: int = 0, num_layers: Optional[int] = None,
                     chunk_layer_begin: int = 0, mode: Optional[int] = None,
                     chunk_ntok: Optional[int] = None, tok_off: int = 0,
                     status=None, chunk_idx=None, chunk_idx_limit: int = 0,
                     num_tokens_dev=None, layout: Optional[PagedKVLayout] = None,
                     chunk_layout=None) -> None:
        from ... import ops

        lay = layout or self.layout
        nl = lay.num_layers - layer_begin if num_layers is None else num_layers
        if chunk is not None and chunk_ntok is None:
            d = 2 if chunk.dim() == 4 else 0
            chunk_ntok = chunk.shape[d]
        ops.native().kv_transfer(
            lay.native(), chunk, chunk_ptrs, chunk_layout or lay.chunk_native(), chunk_ntok or 0,
            tok_off,
            chunk_tokens, chunk_on_device, slots, layer_begin, chunk_layer_begin, nl,
            to_chunk, self._mode() if mode is None else mode,
            status, chunk_idx, chunk_idx_limit, num_tokens_dev)

    def _ensure_stages(self, nbytes: int) -> None:
        if self._stages and self._stages[0].numel() >= nbytes:
            return
        self._stages = [torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                        for _ in range(self.num_stages)]
        self._stage_free = [None] * self.num_stages

    def _slots(self, slot_mapping: torch.Tensor) -> torch.Tensor:
        if slot_mapping.device != self.device:
            slot_mapping = slot_mapping.to(self.device, non_blocking=True)
        if slot_mapping.dtype not in (torch.int32, torch.int64):
            slot_mapping = slot_mapping.long()
        return slot_mapping

    def _contiguous_batch(self, objs, starts, ends) -> bool:
        cs = self.config.chunk_size
        for i, (s, e) in enumerate(zip(starts, ends)):
            if i > 0 and s != ends[i - 1]:
                return False
            if (e - s) != cs and i != len(starts) - 1:
                return False
            if objs[i].get_num_tokens() != e - s:
                return False
        return True

    # -------------------------------------------------------------- store
    @nvtx_range("lmc.batched_from_gpu")
    def batched_from_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                         ends: Sequence[int], slot_mapping: Optional[torch.Tensor] = None,
                         sync: bool = True, **kwargs) -> None:
        if not memory_objs:
            return
        if slot_mapping is None:
            raise ValueError("slot_mapping is required")
        if self.device.type != "cuda":
            for obj, s, e in zip(memory_objs, starts, ends):
                self.layout.gather_ref(obj.tensor, slot_mapping[s:e])
            return
        slots = self._slots(slot_mapping)
        cur = torch.cuda.current_stream(self.device)
        on_device = memory_objs[0].raw_data.is_cuda
        zero_copy = self.config.cpu_transfer_mode == "zero_copy"
        self.store_stream.wait_stream(cur)
        with torch.cuda.stream(self.store_stream):
            if (on_device or zero_copy) and self._contiguous_batch(memory_objs, starts, ends):
                ptrs = torch.tensor([o.data_ptr() for o in memory_objs],
                                    dtype=torch.int64, device=self.device)
                self._native_xfer(None, slots[starts[0]:ends[-1]], True, chunk_ptrs=ptrs,
                                  chunk_tokens=self.config.chunk_size,
                                  chunk_on_device=on_device,
                                  mode=None if on_device else _MODE["simt"])
            elif on_device or zero_copy:
                for obj, s, e in zip(memory_objs, starts, ends):
                    self._native_xfer(obj.tensor, slots[s:e], True,
                                      mode=None if on_device else _MODE["simt"])
            else:
                self._store_via_staging(memory_objs, starts, ends, slots)
        if sync:
            self.store_stream.synchronize()
        nbytes = sum(o.get_size() for o in memory_objs)
        self.stats.inc("from_gpu_bytes", nbytes)

    def _store_via_staging(self, objs, starts, ends, slots) -> None:
        max_bytes = max(o.get_size() for o in objs)
        self._ensure_stages(max_bytes)
        for i, (obj, s, e) in enumerate(zip(objs, starts, ends)):
            k = i % self.num_stages
            ev = self._stage_free[k]
            if ev is not None:
                self.store_stream.wait_event(ev)
            n = obj.get_size()
            stage = self._stages[k][:n].view(obj.get_dtype()).view(obj.get_shape())
            self._native_xfer(stage, slots[s:e], True)
            gathered = torch.cuda.Event()
            gathered.record(self.store_stream)
            self.copy_stream.wait_event(gathered)
            with torch.cuda.stream(self.copy_stream):
                obj.raw_data[:n].copy_(self._stages[k][:n], non_blocking=True)
                done = torch.cuda.Event()
                done.record(self.copy_stream)
            self._stage_free[k] = done
        self.store_stream.wait_stream(self.copy_stream)

    # --------------------------------------------------------------- load
    @nvtx_range("lmc.batched_to_gpu")
    def batched_to_gpu(self, memory_objs: Sequence[MemoryObj], starts: Sequence[int],
                       ends: Sequence[int], slot_mapping: Optional[torch.Tensor] = None,
                       sync: bool = True, **kwargs) -> None:
        if not memory_objs:
            return
        if slot_mapping is None:
            raise ValueError("slot_mapping is required")
        if any(is_proxy(o) and not o.resolved for o in memory_objs):
            self._load_proxies(memory_objs, starts, ends, slot_mapping)
            return
        if self.device.type != "cuda":
            for obj, s, e in zip(memory_objs, starts, ends):
                self.layout.scatter_ref(obj.tensor, slot_mapping[s:e])
            return
        slots = self._slots(slot_mapping)
        cur = torch.cuda.current_stream(self.device)
        on_device = memory_objs[0].raw_data.is_cuda
        zero_copy = self.config.cpu_transfer_mode == "zero_copy"
        self.load_stream.wait_stream(cur)
        with torch.cuda.stream(self.load_stream):
            if (on_device or zero_copy) and self._contiguous_batch(memory_objs, starts, ends):
                ptrs = torch.tensor([o.data_ptr() for o in memory_objs],
                                    dtype=torch.int64, device=self.device)
                self._native_xfer(None, slots[starts[0]:ends[-1]], False, chunk_ptrs=ptrs,
                                  chunk_tokens=self.config.chunk_size,
                                  chunk_on_device=on_device,
                                  mode=None if on_device else _MODE["simt"])
            elif on_device or zero_copy:
                for obj, s, e in zip(memory_objs, starts, ends):
                    self._native_xfer(obj.tensor, slots[s:e], False,
                                      mode=None if on_device else _MODE["simt"])
            else:
                self._load_via_staging(memory_objs, starts, ends, slots)
        cur.wait_stream(self.load_stream)
        if sync:
            self.load_stream.synchronize()
        self.stats.inc("to_gpu_bytes", sum(o.get_size() for o in memory_objs))

    def _load_proxies(self, objs, starts, ends, slot_mapping) -> None:
        """Chunks still on a peer: read them bank by bank into the transfer
        context's bounce buffers and scatter each bank while the next one is
        read (reference npu_connectors.py proxy ping-pong pipeline)."""
        def scatter(batch, s, e):
            self.batched_to_gpu(batch, s, e, slot_mapping, sync=False)
            if self.device.type != "cuda":
                return None
            ev = torch.cuda.Event()
            ev.record(self.load_stream)
            return ev

        plain = [i for i, o in enumerate(objs) if not is_proxy(o)]
        if plain:
            self.batched_to_gpu([objs[i] for i in plain], [starts[i] for i in plain],
                                [ends[i] for i in plain], slot_mapping, sync=False)
        px = [i for i, o in enumerate(objs) if is_proxy(o)]
        load_proxies_pipelined([objs[i] for i in px], [starts[i] for i in px],
                               [ends[i] for i in px], scatter)
        if self.device.type == "cuda":
            self.load_stream.synchronize()

    def _load_via_staging(self, objs, starts, ends, slots) -> None:
        max_bytes = max(o.get_size() for o in objs)
        self._ensure_stages(max_bytes)
        for i, (obj, s, e) in enumerate(zip(objs, starts, ends)):
            k = i % self.num_stages
            ev = self._stage_free[k]
            if ev is not None:
                self.copy_stream.wait_event(ev)
            n = obj.get_size()
            with torch.cuda.stream(self.copy_stream):
                self._stages[k][:n].copy_(obj.raw_data[:n], non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(self.copy_stream)
            self.load_stream.wait_event(arrived)
            stage = self._stages[k][:n].view(obj.get_dtype()).view(obj.get_shape())
            self._native_xfer(stage, slots[s:e], False)
            done = torch.cuda.Event()
            done.record(self.load_stream)
            self._stage_free[k] = done

    def close(self) -> None:
        self._stages = []


class VLLMPagedMemLayerwiseGPUConnector(VLLMPagedMemGPUConnector):
    """Layer-by-layer transfers as generators (num_layers + 2 yields).

    The store generator gathers layer l of every chunk when resumed after the
    model wrote layer l's KV; the load generator scatters layer l so the
    model's ``wait_for_layer_load`` for layer l can proceed while l+1 is in
    flight (reference npu_connectors.py:6255-6893).  Chunk objects here are
    per layer: shape ``[2, 1, T, H*D]`` (or ``[1, 1, T, D]`` for MLA).
    """

    def get_shape(self, num_tokens: int) -> torch.Size:
        s = list(self.layout.chunk_shape(num_tokens))
        s[1] = 1
        return torch.Size(s)

    def _layer_layout_native(self):
        if getattr(self, "_ll", None) is None:
            from ... import ops

            rb = self.layout.row_bytes
            if self.layout.fmt.uses_2ltd_chunks:
                params = ([rb[0]] * 2, rb[0], [rb[0]] * 2, [0, 0])
            else:
                params = self.layout.chunk_layout_params()
            self._ll = ops.native().ChunkLayout(*params)
        return self._ll

    def _layer_tables(self, objs_per_layer, starts, ends, stream):
        """Device pointer tables [L, chunks] of every layer's chunk objects,
        uploaded with one copy on ``stream`` (the stream that reads them), when
        the chunks tile the token range (all full except the last): each layer
        then moves in one launch."""
        if self.device.type != "cuda" or not objs_per_layer or not objs_per_layer[0]:
            return None
        if not self._contiguous_batch(objs_per_layer[0], starts, ends):
            return None
        ptrs = torch.tensor([[o.data_ptr() for o in row] for row in objs_per_layer],
                            dtype=torch.int64).pin_memory()
        with torch.cuda.stream(stream):
            return ptrs.to(self.device, non_blocking=True)

    def _xfer_layer(self, objs, starts, ends, slots, layer: int, to_chunk: bool,
                    table=None) -> None:
        if table is not None:
            on_dev = objs[0].raw_data.is_cuda
            self._native_xfer(None, slots[starts[0]:ends[-1]], to_chunk, chunk_ptrs=table[layer],
                              chunk_tokens=self.config.chunk_size, chunk_on_device=on_dev,
                              layer_begin=layer, num_layers=1, chunk_layer_begin=0,
                              mode=None if on_dev else _MODE["simt"],
                              layout=None, chunk_layout=self._layer_layout_native())
            return
        if self.device.type != "cuda":
            for obj, s, e in zip(objs, starts, ends):
                if to_chunk:
                    self.layout.gather_ref(obj.tensor, slots[s:e], layer_begin=layer,
                                           num_layers=1, chunk_layer_begin=0)
                else:
                    self.layout.scatter_ref(obj.tensor, slots[s:e], layer_begin=layer,
                                            num_layers=1, chunk_layer_begin=0)
            return
        from ... import ops

        for obj, s, e in zip(objs, starts, ends):
            t = obj.tensor
            ops.native().kv_transfer(
                self.layout.native(), t, None, self._layer_layout_native(), t.shape[2], 0, 0,
                t.is_cuda, slots[s:e], layer, 0, 1, to_chunk,
                self._mode() if t.is_cuda else _MODE["simt"], None, None, 0, None)

    def batched_from_gpu(self, memory_objs, starts, ends, slot_mapping=None, sync=True,
                         **kwargs) -> Generator[None, None, None]:
        """Generator: yield once, then gather layer l at each resume."""
        objs_per_layer: List[List[MemoryObj]] = memory_objs  # [L][chunks]
        slots = slot_mapping if self.device.type != "cuda" else self._slots(slot_mapping)
        plan = self._staged_plan(objs_per_layer, starts, ends, store=True)
        if plan is not None:
            yield
            for layer in range(self.layout.num_layers):
                self.store_stream.wait_stream(torch.cuda.current_stream(self.device))
                self._staged_store_layer(plan, layer, starts, ends, slots)
                yield
            self.store_stream.wait_stream(self.copy_stream)
            if sync:
                self.store_stream.synchronize()
            return
        table = self._layer_tables(objs_per_layer, starts, ends, self.store_stream)
        yield
        for layer in range(self.layout.num_layers):
            if self.device.type == "cuda":
                self.store_stream.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(self.store_stream):
                    self._xfer_layer(objs_per_layer[layer], starts, ends, slots, layer, True,
                                     table)
            else:
                self._xfer_layer(objs_per_layer[layer], starts, ends, slots, layer, True)
            yield
        if self.device.type == "cuda" and sync:
            self.store_stream.synchronize()

    def _staged_plan(self, objs_per_layer, starts, ends, store: bool = False):
        """Copy-engine plan for host chunk objects.  Loads: each layer's objects
        are copied whole (one coalesced cudaMemcpyAsync batch from pinned
        memory) into the slots of one of two device staging banks, then
        scattered from the bank by one TMA launch through a pointer table of
        its slots.  Stores (``store``): the mirror image, TMA gather into a
        bank then one coalesced device-to-host batch; loads and stores use
        separate banks."""
        if (self.device.type != "cuda" or self.config.cpu_transfer_mode != "copy_engine"
                or not objs_per_layer or not objs_per_layer[0]
                or objs_per_layer[0][0].raw_data.is_cuda
                or not self._contiguous_batch(objs_per_layer[0], starts, ends)):
            return None
        row0 = objs_per_layer[0]
        n = len(row0)
        slot = (max(o.get_size() for o in row0) + 255) // 256 * 256
        need = n * slot
        attr = "_lws" if store else "_lw"
        banks = getattr(self, attr + "_banks", None)
        if banks is None or banks[0].numel() < need:
            banks = [torch.empty(need, dtype=torch.uint8, device=self.device) for _ in range(2)]
            setattr(self, attr + "_banks", banks)
            setattr(self, attr + "_free", [None, None])
        dst = [torch.tensor([b.data_ptr() + i * slot for i in range(n)], dtype=torch.int64)
               for b in banks]
        with torch.cuda.stream(self.store_stream if store else self.load_stream):
            dev_tables = [d.pin_memory().to(self.device, non_blocking=True) for d in dst]
        sizes = torch.tensor([o.get_size() for o in row0], dtype=torch.int64)
        # host addresses are read per layer, when that layer moves: the rows of
        # later layers may still be being fetched from the CPU tier
        return dst, dev_tables, objs_per_layer, sizes

    def _staged_store_layer(self, plan, layer, starts, ends, slots) -> None:
        from ... import ops

        bank_ptrs, dev_tables, objs, sizes = plan
        host = torch.tensor([o.data_ptr() for o in objs[layer]], dtype=torch.int64)
        b = layer & 1
        if self._lws_free[b] is not None:  # the bank's previous copy-out must be done
            self.store_stream.wait_event(self._lws_free[b])
        with torch.cuda.stream(self.store_stream):
            self._native_xfer(None, slots[starts[0]:ends[-1]], True, chunk_ptrs=dev_tables[b],
                              chunk_tokens=self.config.chunk_size, chunk_on_device=True,
                              layer_begin=layer, num_layers=1, chunk_layer_begin=0,
                              chunk_layout=self._layer_layout_native())
            gathered = torch.cuda.Event()
            gathered.record(self.store_stream)
        self.copy_stream.wait_event(gathered)
        with torch.cuda.stream(self.copy_stream):
            ops.native().layerwise_prefill_dma_copy(host, bank_ptrs[b], sizes)
            free = torch.cuda.Event()
            free.record(self.copy_stream)
        self._lws_free[b] = free

    def _staged_load_layer(self, plan, layer, starts, ends, slots) -> None:
        from ... import ops

        dst, dev_tables, objs, sizes = plan
        srcs_l = torch.tensor([o.data_ptr() for o in objs[layer]], dtype=torch.int64)
        b = layer & 1
        if self._lw_free[b] is not None:  # the bank's previous scatter must be done
            self.copy_stream.wait_event(self._lw_free[b])
        with torch.cuda.stream(self.copy_stream):
            ops.native().layerwise_prefill_dma_copy(dst[b], srcs_l, sizes)
            copied = torch.cuda.Event()
            copied.record(self.copy_stream)
        self.load_stream.wait_event(copied)
        with torch.cuda.stream(self.load_stream):
            self._native_xfer(None, slots[starts[0]:ends[-1]], False, chunk_ptrs=dev_tables[b],
                              chunk_tokens=self.config.chunk_size, chunk_on_device=True,
                              layer_begin=layer, num_layers=1, chunk_layer_begin=0,
                              chunk_layout=self._layer_layout_native())
            free = torch.cuda.Event()
            free.record(self.load_stream)
        self._lw_free[b] = free

    def batched_to_gpu(self, memory_objs=None, starts=None, ends=None, slot_mapping=None,
                       sync=True, **kwargs) -> Generator[None, List[List[MemoryObj]], None]:
        """Generator: first ``send`` the per-layer objects, then one layer per resume."""
        objs_per_layer = yield
        slots = slot_mapping if self.device.type != "cuda" else self._slots(slot_mapping)
        plan = self._staged_plan(objs_per_layer, starts, ends)
        if plan is not None:
            for layer in range(self.layout.num_layers):
                self._staged_load_layer(plan, layer, starts, ends, slots)
                torch.cuda.current_stream(self.device).wait_stream(self.load_stream)
                yield
            if sync:
                self.load_stream.synchronize()
            yield
            return
        row0 = objs_per_layer[0] if len(objs_per_layer) else []
        if self.device.type == "cuda" and row0 and row0[0].raw_data.is_cuda and \
                self._contiguous_batch(row0, starts, ends):
            # device-resident chunks (HBM tier): layer l's pointer table is built
            # when layer l moves, so the tiers are asked for layer l's chunks
            # only then (the fetches of later layers overlap earlier copies)
            L = self.layout.num_layers
            host_tbl = torch.empty(L, len(row0), dtype=torch.int64, pin_memory=True)
            rows_np = host_tbl.numpy()
            for layer in range(L):
                rows_np[layer] = [o.data_ptr() for o in objs_per_layer[layer]]
                with torch.cuda.stream(self.load_stream):
                    self._native_xfer(None, slots[starts[0]:ends[-1]], False,
                                      chunk_ptrs=host_tbl[layer].to(self.device,
                                                                    non_blocking=True),
                                      chunk_tokens=self.config.chunk_size,
                                      chunk_on_device=True, layer_begin=layer, num_layers=1,
                                      chunk_layer_begin=0,
                                      chunk_layout=self._layer_layout_native())
                torch.cuda.current_stream(self.device).wait_stream(self.load_stream)
                yield
            if sync:
                self.load_stream.synchronize()
            yield
            return
        table = self._layer_tables(objs_per_layer, starts, ends, self.load_stream)
        for layer in range(self.layout.num_layers):
            if self.device.type == "cuda":
                with torch.cuda.stream(self.load_stream):
                    self._xfer_layer(objs_per_layer[layer], starts, ends, slots, layer, False,
                                     table)
                torch.cuda.current_stream(self.device).wait_stream(self.load_stream)
            else:
                self._xfer_layer(objs_per_layer[layer], starts, ends, slots, layer, False)
            yield
        if self.device.type == "cuda" and sync:
            self.load_stream.synchronize()
        yield


class VLLMBufferLayerwiseGPUConnector(VLLMPagedMemLayerwiseGPUConnector):
    """Layerwise connector used by CacheBlend (reference
    npu_connectors.py:405-786).  For each layer it assembles the retrieved
    chunks into one dense ``[2, T, H*D]`` buffer covering the request's
    token range, re-rotates K from the positions the chunks were stored at
    to their positions in this request (fused RoPE, K8), zeroes the tokens no
    chunk covers (segment separators), exposes the buffer to the blender
    (``get_kv``) and writes it into the paged cache."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.fused_rope = None
        self._bufs = {}

    def get_kv(self, layer_id: int):
        buf = self._bufs[layer_id]
        return buf[0], buf[1]

    def batched_to_gpu(self, memory_objs=None, starts=None, ends=None, slot_mapping=None,
                       sync=True, **kwargs):
        from ...ops import api

        objs_per_layer = yield
        base, stop = starts[0], ends[-1]
        total = stop - base
        dev = self.device
        lay = self.layout
        e = lay.planes[0].row_elems
        new_pos = torch.arange(base, stop, device=dev)
        old_pos = new_pos.clone()
        covered = torch.zeros(total, dtype=torch.bool, device=dev)
        for s, en, o in zip(starts, ends, objs_per_layer[0]):
            cp = o.meta.cached_positions
            old_pos[s - base:en - base] = (cp.to(dev) if cp is not None else
                                           torch.arange(0, en - s, device=dev))
            covered[s - base:en - base] = True
        need_rope = self.fused_rope is not None and not torch.equal(old_pos, new_pos)
        slots = slot_mapping[base:stop].to(dev).clone()
        slots[~covered] = -1
        self._bufs = {}
        for layer in range(lay.num_layers):
            buf = torch.zeros(2, total, e, dtype=lay.dtype, device=dev)
            for s, en, o in zip(starts, ends, objs_per_layer[layer]):
                buf[:, s - base:en - base] = o.tensor[:, 0].to(dev, non_blocking=True)
            if need_rope:
                self.fused_rope(old_pos, new_pos, buf[0])
            self._bufs[layer] = buf
            api.single_layer_kv_transfer(buf, lay, layer, slots, False)
            yield
        if dev.type == "cuda" and sync:
            torch.cuda.current_stream(dev).synchronize()
        yield


class _SGLangPools:
    """SGLang caches: ``[K_all, V_all]`` each ``[L, NB, BS, H, D]``, per-layer
    token pools ``[L, size, H, D]`` (page size 1), or per-layer (K, V)
    tuples (reference npu_connectors.py:8093-8376)."""

    def register_kv_caches(self, kvcaches, fmt=None) -> None:
        if isinstance(kvcaches, (list, tuple)) and len(kvcaches) == 2 and \
                isinstance(kvcaches[0], torch.Tensor) and kvcaches[0].dim() == 4:
            k, v = kvcaches  # per-layer token pool [L, size, H, D] -> block dim of 1
            kvcaches = [k.unsqueeze(2), v.unsqueeze(2)]
        super().register_kv_caches(list(kvcaches), fmt or KVCacheFormat.SEPARATE_KV)


class SGLangGPUConnector(_SGLangPools, VLLMPagedMemGPUConnector):
    def __init__(self, config=None, device=None, use_mla=False, layerwise=False, **kw):
        VLLMPagedMemGPUConnector.__init__(self, config, device=device, use_mla=use_mla, **kw)
        self.layerwise = layerwise


class SGLangLayerwiseGPUConnector(_SGLangPools, VLLMPagedMemLayerwiseGPUConnector):
    def __init__(self, config=None, device=None, use_mla=False, **kw):
        VLLMPagedMemLayerwiseGPUConnector.__init__(self, config, device=device, use_mla=use_mla,
                                                   **kw)
        self.layerwise = True
