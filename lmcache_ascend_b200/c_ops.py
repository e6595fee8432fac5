"""The reference's native op table with its call signatures.

``lmcache_ascend.c_ops`` (reference csrc/pybind.cpp:243-483) takes raw
pointer tables, format codes and hidden sizes.  This module accepts those
argument lists and runs them on this framework's sm_100a kernels, so code
written against ``c_ops`` can switch imports:

    from lmcache_ascend_b200 import c_ops as lmc_ops

``ops.api`` is the native surface (paged caches described once by a layout
object); the functions here build that description from the arguments of
each call (cached per pointer table) and forward.

Pointer tables follow the reference connector's convention
(lmcache_ascend/v1/npu_connector/npu_connectors.py:862-935): per layer, the
base address of each plane of the paged cache, layer-major:

* ``kvcache_format_raw`` 1 (MERGED_KV): one pointer per layer to a
  ``[2, page_buffer_size, hidden]`` two-major cache (K then V);
* 2 (SEPARATE_KV): ``k_l, v_l`` per layer, each ``[page_buffer_size, hidden]``;
* 3 (MLA_KV): latent (``k_hidden_dims``) and rope (``v_hidden_dims``) planes;
* 4 (DSA_KV): latent, rope and indexer (``dsa_hidden_dims``) planes.

``page_buffer_size`` is the number of slots (blocks x block size).  MLA and
DSA chunks are ``[1, L, T, sum of the planes' dims]``; the others are
``[2, L, T, hidden]``.  ``direction`` True moves paged -> chunk.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from .ops import api, native

MERGED_KV, SEPARATE_KV, MLA_KV, DSA_KV = 1, 2, 3, 4

_layouts: Dict[tuple, "_TableLayout"] = {}


class _TableLayout:
    """Paged-cache description built from a pointer table (one block that
    holds every slot: planes are contiguous ``[page_buffer_size, row]``)."""

    def __init__(self, ptrs: torch.Tensor, planes: int, page_buffer_size: int,
                 row_bytes: List[int], device: torch.device, two_ltd: bool):
        host = ptrs.detach().to("cpu", torch.int64).view(-1)
        if host.numel() % planes:
            raise ValueError("pointer table length is not a multiple of the planes per layer")
        self.num_layers = host.numel() // planes
        self.row_bytes = row_bytes
        self.device = device
        self.two_ltd = two_ltd
        self._host = host
        self._native = None
        self._chunk = None
        self._pbs = int(page_buffer_size)

    def native(self):
        if self._native is None:
            table = self._host.to(self.device)
            rb = self.row_bytes
            self._native = native().PagedLayout(table, [self._pbs * r for r in rb], list(rb),
                                                list(rb), self._pbs, self._pbs)
            self._native.set_bases_aligned(bool((self._host % 16 == 0).all()))
        return self._native

    def chunk_native(self):
        if self._chunk is None:
            rb, L = self.row_bytes, self.num_layers
            if self.two_ltd:
                self._chunk = native().ChunkLayout([L * rb[0]] * 2, rb[0], [rb[0]] * 2, [0, 0])
            else:
                row = sum(rb)
                offs = [sum(rb[:p]) for p in range(len(rb))]
                self._chunk = native().ChunkLayout([0] * len(rb), row, [row] * len(rb), offs)
        return self._chunk


def _layout(key_value: torch.Tensor, key_value_ptrs: torch.Tensor, device, page_buffer_size,
            use_mla: bool, fmt: int, k_dims: int, v_dims: int, dsa_dims: int) -> _TableLayout:
    es = key_value.element_size()
    if use_mla or fmt in (MLA_KV, DSA_KV):
        dims = [k_dims, v_dims] + ([dsa_dims] if fmt == DSA_KV else [])
        if fmt not in (MLA_KV, DSA_KV) or not all(dims):
            dims = [int(key_value.shape[-1])]  # one latent plane
        rb, two_ltd = [d * es for d in dims], False
    else:
        rb, two_ltd = [int(key_value.shape[-1]) * es] * 2, True
    planes = len(rb) if fmt in (SEPARATE_KV, MLA_KV, DSA_KV) else 1
    # keyed by the table's values (a small copy to the host): a table freed
    # and reallocated at the same address must not reuse a stale description
    ptrs = key_value_ptrs.detach().to("cpu", torch.int64).view(-1)
    key = (tuple(ptrs.tolist()), int(page_buffer_size), tuple(rb), planes, two_ltd)
    lay = _layouts.get(key)
    if lay is None:
        if planes == 1 and two_ltd:
            # merged two-major: V follows K inside the same allocation
            plane = int(page_buffer_size) * rb[0]
            ptrs = torch.stack([ptrs, ptrs + plane], dim=1).view(-1)
            planes = 2
        lay = _TableLayout(ptrs, planes, page_buffer_size, rb, torch.device(device), two_ltd)
        _layouts[key] = lay
    return lay


def multi_layer_kv_transfer(key_value: torch.Tensor, key_value_ptrs: torch.Tensor,
                            slot_mapping: torch.Tensor, paged_memory_device,
                            page_buffer_size: int, direction: bool, use_mla: bool = False,
                            kvcache_format_raw: int = MERGED_KV, k_hidden_dims: int = 0,
                            v_hidden_dims: int = 0, dsa_hidden_dims: int = 0) -> None:
    """Every layer of a chunk <-> the paged cache in one launch
    (reference csrc/mem_kernels.cpp:75-111)."""
    lay = _layout(key_value, key_value_ptrs, paged_memory_device, page_buffer_size, use_mla,
                  kvcache_format_raw, k_hidden_dims, v_hidden_dims, dsa_hidden_dims)
    on_dev = key_value.is_cuda
    api._xfer(lay, key_value, slot_mapping.to(lay.device), direction, chunk_on_device=on_dev,
              mode=api.MODE_AUTO if on_dev else api.MODE_SIMT)


def fused_multi_layer_kv_transfer(key_value: torch.Tensor, staging_cache: torch.Tensor,
                                  key_value_ptrs: torch.Tensor, slot_mapping: torch.Tensor,
                                  paged_memory_device, page_buffer_size: int, direction: bool,
                                  use_mla: bool = False, kvcache_format_raw: int = MERGED_KV,
                                  k_hidden_dims: int = 0, v_hidden_dims: int = 0,
                                  dsa_hidden_dims: int = 0) -> None:
    """Host chunk <-> paged cache through a device staging buffer
    (reference csrc/mem_kernels.cpp:113-213)."""
    lay = _layout(key_value, key_value_ptrs, paged_memory_device, page_buffer_size, use_mla,
                  kvcache_format_raw, k_hidden_dims, v_hidden_dims, dsa_hidden_dims)
    need = key_value.numel() * key_value.element_size()
    if staging_cache.numel() * staging_cache.element_size() < need:
        raise ValueError("staging cache smaller than the chunk")
    api.fused_multi_layer_kv_transfer(key_value, staging_cache, lay,
                                      slot_mapping.to(lay.device), direction)


def multi_layer_kv_transfer_unilateral(*args, **kwargs):
    return api.multi_layer_kv_transfer_unilateral(*args, **kwargs)


# ------------------------------------------------------ tensor-argument ops
def _kv_list(vllm_kv_caches, fmt: int, two_major: bool):
    """A one-layer ``vllm_kv_caches`` argument as the [layer][plane] nesting a
    ``PagedKVLayout`` takes (merged: one [2, NB, BS, H, D] or
    [NB, 2, BS, H, D] tensor; separate / MLA / DSA: a list of planes)."""
    from .v1.kv_format import PagedKVLayout

    if isinstance(vllm_kv_caches, torch.Tensor):
        t = vllm_kv_caches
        if fmt == MERGED_KV and t.dim() == 5:
            planes = [t[0], t[1]] if two_major else [t[:, 0], t[:, 1]]
        else:
            planes = [t]
    else:
        planes = list(vllm_kv_caches)
    key = tuple((p.data_ptr(), tuple(p.shape), tuple(p.stride())) for p in planes)
    lay = _layouts.get(key)
    if lay is None:
        if len(_layouts) > 256:  # descriptions hold views of the caches
            _layouts.clear()
        lay = PagedKVLayout([tuple(planes)] if len(planes) > 1 else [planes[0]],
                            use_mla=len(planes) != 2 or fmt in (MLA_KV, DSA_KV))
        _layouts[key] = lay
    return lay


def single_layer_kv_transfer(lmc_key_value_cache: torch.Tensor, vllm_kv_caches,
                             slot_mapping: torch.Tensor, direction: bool,
                             kvcache_format_raw: int = SEPARATE_KV, token_major: bool = False,
                             vllm_two_major: bool = False, k_hidden_dims: int = 0,
                             v_hidden_dims: int = 0, dsa_hidden_dims: int = 0) -> None:
    """One layer between a per-layer LMCache buffer ([T, 2, E] token-major,
    else [2, T, E]) and that layer's paged cache (reference
    csrc/mem_kernels.cpp:265-334, pybind.cpp:33-43)."""
    lay = _kv_list(vllm_kv_caches, kvcache_format_raw, vllm_two_major)
    api.single_layer_kv_transfer(lmc_key_value_cache, lay, 0, slot_mapping.to(lay.device),
                                 direction, token_major)


def load_and_reshape_flash(key_value: torch.Tensor, key_cache: torch.Tensor,
                           value_cache: torch.Tensor, slot_mapping: torch.Tensor,
                           layer_idx: int) -> None:
    """Layer ``layer_idx`` of a [2, L, T, H*D] chunk -> a flash-layout layer
    (reference csrc/mem_kernels.cpp:1341-1389)."""
    lay = _kv_list([key_cache, value_cache], SEPARATE_KV, False)
    api._xfer(lay, key_value, slot_mapping.to(lay.device), False,
              chunk_on_device=key_value.is_cuda, layer_begin=0, num_layers=1,
              chunk_layer_begin=layer_idx,
              mode=api.MODE_AUTO if key_value.is_cuda else api.MODE_SIMT,
              chunk_layout=_chunk_2ltd(lay, key_value.shape[1]))


def reshape_and_cache_back_flash(key_value: torch.Tensor, key_cache: torch.Tensor,
                                 value_cache: torch.Tensor, slot_mapping: torch.Tensor,
                                 layer_idx: int) -> None:
    """A flash-layout layer -> layer ``layer_idx`` of a [2, L, T, H*D] chunk
    (reference csrc/mem_kernels.cpp:1391-1440)."""
    lay = _kv_list([key_cache, value_cache], SEPARATE_KV, False)
    api._xfer(lay, key_value, slot_mapping.to(lay.device), True,
              chunk_on_device=key_value.is_cuda, layer_begin=0, num_layers=1,
              chunk_layer_begin=layer_idx,
              mode=api.MODE_AUTO if key_value.is_cuda else api.MODE_SIMT,
              chunk_layout=_chunk_2ltd(lay, key_value.shape[1]))


def _chunk_2ltd(lay, chunk_layers: int):
    rb = lay.row_bytes[0]
    return native().ChunkLayout([chunk_layers * rb] * 2, rb, [rb] * 2, [0, 0])


def rotary_embedding_k_fused(old_positions: torch.Tensor, new_positions: torch.Tensor,
                             key: torch.Tensor, head_size: int, cos_sin_cache: torch.Tensor,
                             is_neox: bool) -> None:
    """In-place K re-rotation (reference csrc/pos_kernels.cpp:158)."""
    api.rotary_embedding_k_fused(old_positions, new_positions, key, head_size, cos_sin_cache,
                                 is_neox)


def layerwise_prefill_dma_copy(copies: Sequence[tuple], device_to_host: bool = False) -> None:
    """``[(dst, src, bytes), ...]`` copies on the current stream (reference
    csrc/pybind.cpp:295-311); ``device_to_host`` only names the direction."""
    if not copies:
        return
    d, s, n = zip(*copies)
    native().layerwise_prefill_dma_copy(torch.tensor(d, dtype=torch.int64),
                                        torch.tensor(s, dtype=torch.int64),
                                        torch.tensor(n, dtype=torch.int64))


calculate_cdf = api.calculate_cdf
encode_fast_new = api.encode_fast_new
decode_fast_new = api.decode_fast_new
decode_fast_prefsum = api.decode_fast_prefsum
get_gpu_pci_bus_id = api.get_gpu_pci_bus_id


def __getattr__(name: str):
    """Allocators and registry calls (``alloc_pinned_ptr``, ``free_pinned_ptr``,
    ``alloc_pinned_numa_ptr``, ``alloc_shm_pinned_ptr``, ``attach_shm_pinned_ptr``,
    ``unlink_shm``, ...) come straight from the native module, which uses the
    reference's names."""
    mod = native()
    if hasattr(mod, name):
        return getattr(mod, name)
    raise AttributeError(name)
