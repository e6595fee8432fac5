"""Public op surface under the reference's op names.

Each function takes the same kind of arguments as the reference's pybind
op (csrc/pybind.cpp:243-483) where that makes sense on CUDA, and dispatches:
CUDA tensors -> the native sm_100a kernels (mandatory, fails loudly if the
extension is missing); CPU tensors -> the PyTorch oracles.  Paged caches are
described once by ``PagedKVLayout`` (``v1/kv_format.py``).

Ops here:
  multi_layer_kv_transfer, fused_multi_layer_kv_transfer,
  single_layer_kv_transfer, batched_fused_single_layer_kv_transfer,
  sparse_single_layer_kv_transfer, batched_fused_sparse_single_layer_kv_transfer,
  dense_mla_dsa_batched_direct_kv_transfer (multi-chunk pointer table),
  sparse_graph_kv_transfer (device-side count, CUDA-graph capturable),
  load_and_reshape_flash, reshape_and_cache_back_flash,
  IndexerC8State / IndexerC8GroupState / indexer_c8_transfer_prepared,
  calculate_cdf, encode_fast_new, decode_fast_prefsum,
  rotary_embedding_k_fused, rotary_embedding_k_fused_layers (every layer in one
  launch), layerwise_prefill_dma_copy, get_gpu_pci_bus_id.
The reference's raw-pointer call signatures are in ``lmcache_ascend_b200.c_ops``.
"""

from __future__ import annotations

from typing import Tuple, List, Optional, Sequence

import torch

from . import native, reference as R

MODE_AUTO, MODE_TMA, MODE_SIMT = 0, 1, 2


def _xfer(layout, chunk, slots, to_chunk, *, chunk_ptrs=None, chunk_tokens=0,
          chunk_on_device=True, layer_begin=0, num_layers=None, chunk_layer_begin=0,
          chunk_layout=None, tok_off=0, chunk_idx=None, chunk_idx_limit=0,
          num_tokens_dev=None, mode=MODE_AUTO, status=None):
    nl = layout.num_layers - layer_begin if num_layers is None else num_layers
    ntok = 0
    if chunk is not None:
        ntok = chunk.shape[2] if chunk.dim() == 4 else chunk.shape[0]
    native().kv_transfer(layout.native(), chunk, chunk_ptrs,
                         chunk_layout or layout.chunk_native(), ntok, tok_off, chunk_tokens,
                         chunk_on_device, slots, layer_begin, chunk_layer_begin, nl, to_chunk,
                         mode, status, chunk_idx, chunk_idx_limit, num_tokens_dev)


# ----------------------------------------------------------------- K1 / N2
def multi_layer_kv_transfer(key_value: torch.Tensor, layout, slot_mapping: torch.Tensor,
                            direction: bool, mode: int = MODE_AUTO) -> None:
    """All layers between ``key_value`` (chunk [2|1, L, T, E], device or
    pinned host) and the paged cache.  ``direction`` True = paged -> chunk
    (from_gpu), False = chunk -> paged (reference mem_kernels.cpp:75-111)."""
    if layout.device.type != "cuda":
        (layout.gather_ref if direction else layout.scatter_ref)(key_value, slot_mapping)
        return
    on_dev = key_value.is_cuda
    _xfer(layout, key_value, slot_mapping, direction, chunk_on_device=on_dev,
          mode=mode if on_dev else MODE_SIMT)


def fused_multi_layer_kv_transfer(key_value: torch.Tensor, staging: torch.Tensor, layout,
                                  slot_mapping: torch.Tensor, direction: bool,
                                  mode: int = MODE_AUTO) -> None:
    """Pinned host chunk <-> paged cache through a device staging buffer
    (gather/scatter + one copy-engine transfer; reference mem_kernels.cpp:113-213)."""
    native().fused_multi_layer_kv_transfer(key_value, staging, layout.native(),
                                           layout.chunk_native(), slot_mapping, direction, mode)


# ----------------------------------------------------------------- K2 / N3
_layer_layouts = {}


def _single_layer_layout(layout, token_major: bool):
    key = (id(layout), token_major)
    if key not in _layer_layouts:
        rb = layout.row_bytes
        if token_major:  # [T, P, E] rows
            row = sum(rb)
            offs = [sum(rb[:p]) for p in range(len(rb))]
            _layer_layouts[key] = native().ChunkLayout([0] * len(rb), row, [row] * len(rb), offs)
        elif layout.fmt.uses_2ltd_chunks:  # [2, T, E]
            _layer_layouts[key] = native().ChunkLayout([rb[0]] * 2, rb[0], [rb[0]] * 2, [0, 0])
        else:  # [1, T, sum E] (MLA rows)
            _layer_layouts[key] = native().ChunkLayout(*layout.chunk_layout_params())
    return _layer_layouts[key]


def single_layer_kv_transfer(lmc_kv: torch.Tensor, layout, layer: int,
                             slot_mapping: torch.Tensor, direction: bool,
                             token_major: bool = False, mode: int = MODE_AUTO) -> None:
    """One layer between a per-layer buffer ([T, P, E] token-major, else
    [P, T, E]) and the paged cache (reference mem_kernels.cpp:265-334)."""
    if layout.device.type != "cuda":
        chunk = lmc_kv.transpose(0, 1) if token_major else lmc_kv
        c4 = chunk.unsqueeze(1)
        (layout.gather_ref if direction else layout.scatter_ref)(
            c4, slot_mapping, layer_begin=layer, num_layers=1, chunk_layer_begin=0)
        return
    ntok = lmc_kv.shape[0] if token_major else lmc_kv.shape[1]
    native().kv_transfer(layout.native(), lmc_kv, None, _single_layer_layout(layout, token_major),
                         ntok, 0, 0, lmc_kv.is_cuda, slot_mapping, layer, 0, 1, direction,
                         mode if lmc_kv.is_cuda else MODE_SIMT, None, None, 0, None)


def batched_fused_single_layer_kv_transfer(lmc_kvs: Sequence[torch.Tensor], layout, layer: int,
                                           slot_mappings: Sequence[torch.Tensor],
                                           direction: bool, token_major: bool = False) -> None:
    for kv, sm in zip(lmc_kvs, slot_mappings):
        single_layer_kv_transfer(kv, layout, layer, sm, direction, token_major)


# ----------------------------------------------------------------- K3 / N4
def sparse_single_layer_kv_transfer(staging: torch.Tensor, layout, layer: int,
                                    slot_mapping_packed: torch.Tensor,
                                    selected_token_idx: torch.Tensor,
                                    token_major: bool = False) -> None:
    """paged[slot_mapping_packed[i]] = staging[selected_token_idx[i]] for one
    layer (reference mem_kernels.h:216-218: packed, no -1 holes)."""
    ntok = staging.shape[0] if token_major else staging.shape[1]
    if layout.device.type != "cuda":
        rows = staging.index_select(0 if token_major else 1, selected_token_idx.long().cpu())
        single_layer_kv_transfer(rows, layout, layer, slot_mapping_packed, False, token_major)
        return
    idx = selected_token_idx.to(slot_mapping_packed.dtype)
    native().kv_transfer(layout.native(), staging, None, _single_layer_layout(layout, token_major),
                         ntok, 0, 0, True, slot_mapping_packed, layer, 0, 1, False, MODE_AUTO,
                         None, idx, ntok, None)


def batched_fused_sparse_single_layer_kv_transfer(stagings, layout, layer, slot_mappings,
                                                  selected, token_major=False) -> None:
    for s, sm, sel in zip(stagings, slot_mappings, selected):
        sparse_single_layer_kv_transfer(s, layout, layer, sm, sel, token_major)


# ----------------------------------------------------------------- K4 / N5
def dense_mla_dsa_batched_direct_kv_transfer(chunks: Sequence[torch.Tensor], layout,
                                             slot_mapping: torch.Tensor, chunk_size: int,
                                             direction: bool) -> None:
    """All layers of N chunk objects (host-pinned or device) in ONE launch
    through a device pointer table; token t lives in chunk t // chunk_size
    (reference mem_kernels.cpp:1036-1307, the 'direct' staging-free path)."""
    if layout.device.type != "cuda":
        s = 0
        for c in chunks:
            n = c.shape[2]
            (layout.gather_ref if direction else layout.scatter_ref)(c, slot_mapping[s:s + n])
            s += n
        return
    on_dev = chunks[0].is_cuda
    ptrs = torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64, device=layout.device)
    _xfer(layout, None, slot_mapping, direction, chunk_ptrs=ptrs, chunk_tokens=chunk_size,
          chunk_on_device=on_dev, mode=MODE_AUTO if on_dev else MODE_SIMT)


class DirectTransferState:
    """A fixed list of chunk objects with its device pointer table built once
    (the process-owned state of the reference's ``_prepared`` direct entry
    points, mem_kernels.cpp:1221-1307); reuse it across calls that move the
    same chunks."""

    def __init__(self, chunks: Sequence[torch.Tensor], layout, chunk_size: int):
        if not chunks:
            raise ValueError("direct transfer needs at least one chunk")
        self.layout = layout
        self.chunk_size = int(chunk_size)
        self.chunks = list(chunks)
        self.on_device = chunks[0].is_cuda
        self.ptrs = torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64,
                                 device=layout.device)


_DIRECT_CACHE: "dict" = {}


def dense_mla_dsa_batched_direct_kv_transfer_prepared(state: DirectTransferState,
                                                      slot_mapping: torch.Tensor,
                                                      direction: bool) -> None:
    if state.layout.device.type != "cuda":
        dense_mla_dsa_batched_direct_kv_transfer(state.chunks, state.layout, slot_mapping,
                                                 state.chunk_size, direction)
        return
    _xfer(state.layout, None, slot_mapping, direction, chunk_ptrs=state.ptrs,
          chunk_tokens=state.chunk_size, chunk_on_device=state.on_device,
          mode=MODE_AUTO if state.on_device else MODE_SIMT)


def dense_mla_dsa_batched_direct_kv_transfer_fast(chunks: Sequence[torch.Tensor], layout,
                                                  slot_mapping: torch.Tensor, chunk_size: int,
                                                  direction: bool) -> None:
    """Like the batched direct transfer, with the pointer table cached per
    (layout, chunk addresses) (reference ``_fast``: cached per-layer state)."""
    key = (id(layout), chunk_size, tuple(c.data_ptr() for c in chunks))
    st = _DIRECT_CACHE.get(key)
    if st is None or st.layout is not layout:
        if len(_DIRECT_CACHE) >= 256:
            _DIRECT_CACHE.clear()
        st = _DIRECT_CACHE[key] = DirectTransferState(chunks, layout, chunk_size)
    dense_mla_dsa_batched_direct_kv_transfer_prepared(st, slot_mapping, direction)


def dense_mla_dsa_group_direct_kv_transfer_fast(chunks: Sequence[torch.Tensor], group_layout,
                                                slot_mapping: torch.Tensor, chunk_size: int,
                                                direction: bool) -> None:
    """Every layer of one layer group (a layout over the group's layers) in one
    launch (reference dense_mla_dsa_group_direct_kv_transfer_fast)."""
    dense_mla_dsa_batched_direct_kv_transfer_fast(chunks, group_layout, slot_mapping,
                                                  chunk_size, direction)


def mla_dsa_sparse_multi_chunk_kv_transfer(chunks: Sequence[torch.Tensor], layout,
                                           slot_mapping_packed: torch.Tensor,
                                           selected_token_idx: torch.Tensor,
                                           chunk_size: int) -> None:
    """paged[slot_mapping_packed[i]] = token selected_token_idx[i] of the chunk
    sequence (token t in chunk t // chunk_size), all layers, straight from
    pinned host or device chunks (reference mem_kernels.h:82-154 sparse
    multi-chunk kernels)."""
    if layout.device.type != "cuda":
        full = torch.cat(list(chunks), dim=2)
        rows = full.index_select(2, selected_token_idx.long().cpu())
        layout.scatter_ref(rows, slot_mapping_packed)
        return
    on_dev = chunks[0].is_cuda
    ptrs = torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64, device=layout.device)
    idx = selected_token_idx.to(layout.device, slot_mapping_packed.dtype)
    _xfer(layout, None, slot_mapping_packed.to(layout.device), False, chunk_ptrs=ptrs,
          chunk_tokens=chunk_size, chunk_on_device=on_dev, chunk_idx=idx,
          chunk_idx_limit=len(chunks) * chunk_size,
          mode=MODE_AUTO if on_dev else MODE_SIMT)


def multi_layer_kv_transfer_unilateral(*args, **kwargs):
    raise NotImplementedError("multi_layer_kv_transfer_unilateral is not implemented "
                              "(it is not in the reference either)")


# ----------------------------------------------------------------- K5 / N7
def sparse_graph_kv_transfer(staging: torch.Tensor, layout, layer: int,
                             slot_mapping: torch.Tensor, selected_token_idx: torch.Tensor,
                             active_count: torch.Tensor, token_major: bool = True) -> None:
    """CUDA-graph capturable sparse copy: every input lives in device memory
    and the number of active entries is read on the device from
    ``active_count`` (int32 [1]), so one captured graph replays for any count
    up to the buffers' capacity; out-of-range entries are skipped (reference
    csrc/graph/sparse_graph_kernel.cpp:20-53)."""
    ntok = staging.shape[0] if token_major else staging.shape[1]
    idx = selected_token_idx.to(slot_mapping.dtype) if selected_token_idx.dtype != \
        slot_mapping.dtype else selected_token_idx
    native().kv_transfer(layout.native(), staging, None, _single_layer_layout(layout, token_major),
                         ntok, 0, 0, True, slot_mapping, layer, 0, 1, False, MODE_SIMT,
                         None, idx, ntok, active_count)


# ----------------------------------------------------------------- N6
def load_and_reshape_flash(key_value: torch.Tensor, layout, layer: int,
                           slot_mapping: torch.Tensor) -> None:
    """[2, L, T, H*D] buffer, layer ``layer`` -> separate K/V paged caches
    (reference mem_kernels.cpp:1341-1440)."""
    if layout.device.type != "cuda":
        layout.scatter_ref(key_value, slot_mapping, layer_begin=layer, num_layers=1,
                           chunk_layer_begin=layer)
        return
    _xfer(layout, key_value, slot_mapping, False, layer_begin=layer, num_layers=1,
          chunk_layer_begin=layer, chunk_on_device=key_value.is_cuda)


def reshape_and_cache_back_flash(key_value: torch.Tensor, layout, layer: int,
                                 slot_mapping: torch.Tensor) -> None:
    if layout.device.type != "cuda":
        layout.gather_ref(key_value, slot_mapping, layer_begin=layer, num_layers=1,
                          chunk_layer_begin=layer)
        return
    _xfer(layout, key_value, slot_mapping, True, layer_begin=layer, num_layers=1,
          chunk_layer_begin=layer, chunk_on_device=key_value.is_cuda)


# ----------------------------------------------------------------- K6 / N8
C8_BLOCK = 128
C8_KEY_BYTES = 128
C8_SCALE_BYTES = 2


class IndexerC8State:
    """One layer of the DSA lightning-indexer cache in C8 form: int8 keys
    [NB, 128, 1, 128] + fp16 scales [NB, 128, 1, 1] (or floating keys alone),
    with an optional physical block factor (logical block b at physical block
    b * factor) or block permutation map (reference csrc/indexer_c8.cpp:12-45)."""

    def __init__(self, keys: torch.Tensor, scales: Optional[torch.Tensor] = None,
                 slot_factor: int = 1, block_map: Optional[torch.Tensor] = None):
        quantized = keys.dtype == torch.int8
        if quantized and (scales is None or scales.dtype != torch.float16):
            raise ValueError("int8 indexer keys need float16 scales")
        if not quantized and (scales is not None or keys.dtype not in (torch.float16,
                                                                          torch.bfloat16)):
            raise ValueError("floating indexer keys come without scales")
        if keys.dim() != 4 or keys.shape[1] != C8_BLOCK or keys.shape[2] != 1 or \
                keys.shape[3] != 128 or not keys.is_contiguous():
            raise ValueError("indexer keys must be contiguous [NB, 128, 1, 128]")
        if slot_factor not in (1, 2) or (slot_factor == 2 and not quantized) or \
                keys.shape[0] % slot_factor:
            raise ValueError("invalid physical block factor")
        if block_map is not None and (slot_factor != 1 or block_map.numel() != keys.shape[0]
                                      or block_map.dtype != torch.int32):
            raise ValueError("block map must be int32 [NB] with factor 1")
        self.keys, self.scales = keys, scales
        self.slot_factor, self.block_map = slot_factor, block_map
        self.key_bytes = 128 * keys.element_size()
        self.cache_slots = keys.shape[0] * C8_BLOCK // slot_factor
        self.device = keys.device

    def physical_slots(self, slots: torch.Tensor) -> torch.Tensor:
        s = slots.long()
        bad = (s < 0) | (s >= self.cache_slots)
        if self.block_map is not None:
            phys = self.block_map.long()[(s // C8_BLOCK).clamp(0, self.keys.shape[0] - 1)] \
                * C8_BLOCK + s % C8_BLOCK
        else:
            phys = s + (s // C8_BLOCK) * (self.slot_factor - 1) * C8_BLOCK
        return torch.where(bad, torch.full_like(phys, -1), phys)


class IndexerC8GroupState:
    """All layers of one indexer group, described as one paged layout with a
    key plane and (C8) a scale plane, so a whole group moves in one launch
    (reference csrc/indexer_c8.cpp:47-70)."""

    def __init__(self, states: List[IndexerC8State]):
        if not states:
            raise ValueError("C8 group must contain at least one layer")
        s0 = states[0]
        for s in states:
            if s.device != s0.device or s.cache_slots != s0.cache_slots or \
                    s.key_bytes != s0.key_bytes or (s.scales is None) != (s0.scales is None) \
                    or s.slot_factor != s0.slot_factor:
                raise ValueError("C8 group layers must share device, capacity and format")
        self.states = states
        self.quantized = s0.scales is not None
        self.num_layers = len(states)
        self.key_bytes = s0.key_bytes
        self.row_bytes = [self.key_bytes] + ([C8_SCALE_BYTES] if self.quantized else [])
        self.device = s0.device
        self._native = None
        self._chunk = None

    def packet_bytes(self, count: int) -> int:
        """Bytes of all layers' packets for ``count`` tokens:
        per layer [count * key_bytes keys | count * 2 scale bytes]."""
        return self.num_layers * count * sum(self.row_bytes)

    def native(self):
        if self._native is None:
            ptrs = []
            for s in self.states:
                ptrs.append(s.keys.data_ptr())
                if self.quantized:
                    ptrs.append(s.scales.data_ptr())
            table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
            self._planes = table
            self._aligned = all(p % 16 == 0 for p in ptrs)
            blk = [C8_BLOCK * self.key_bytes] + ([C8_BLOCK * C8_SCALE_BYTES] if self.quantized
                                                 else [])
            slot = self.row_bytes
            nslots = self.states[0].keys.shape[0] * C8_BLOCK
            self._native = native().PagedLayout(table, blk, slot, self.row_bytes, C8_BLOCK, nslots)
            self._native.set_bases_aligned(all(p % 16 == 0 for p in ptrs))
            row = sum(self.row_bytes)
            # per layer: keys then scales; plane 1 starts after count * key_bytes
            self._chunk = native().ChunkLayout([0, self.key_bytes][:len(self.row_bytes)], row,
                                               self.row_bytes, [0] * len(self.row_bytes))
        return self._native

    def chunk_layout(self):
        self.native()
        return self._chunk

    def packet_table(self, addrs: List[int]) -> torch.Tensor:
        """Device int64 table of packet addresses, uploaded without a host
        synchronisation (pinned source) and kept for repeated packet sets."""
        key = tuple(addrs)
        cache = self.__dict__.setdefault("_packet_tables", {})
        t = cache.get(key)
        if t is None:
            if len(cache) >= 64:
                cache.clear()
            host = torch.tensor(addrs, dtype=torch.int64)
            if self.device.type == "cuda":
                host = host.pin_memory()
            t = cache[key] = host.to(self.device, non_blocking=True)
        return t


def indexer_c8_transfer_prepared(group: IndexerC8GroupState, packets: Sequence[torch.Tensor],
                                 slot_mapping: torch.Tensor, chunk_capacity: int,
                                 from_gpu: bool) -> None:
    """Paged C8 indexer cache <-> per-chunk packets (one packet tensor per
    chunk holding every layer; token t of the request is row t % capacity of
    packet t // capacity).  Runs of contiguous slots move as single copies;
    the logical -> physical slot map (factor / block permutation) is applied
    first (reference csrc/indexer_c8.cpp:126-185, kernel :28-150)."""
    group.native()
    addrs = [p.data_ptr() for p in packets]
    if packets[0].is_cuda and group._aligned and all(a % 16 == 0 for a in addrs):
        # device packets: the C8 kernel maps the logical slots itself, stages
        # them once per chunk, and moves 16-byte vectors over the key plane
        # and a 2-byte copy per scale; one launch, no host synchronisation
        s0 = group.states[0]
        slots = slot_mapping.to(group.device, non_blocking=True)
        if slots.dtype not in (torch.int32, torch.int64):
            slots = slots.long()
        native().c8_copy(group._planes, slots, group.packet_table(addrs), chunk_capacity,
                         group.num_layers, group.key_bytes, s0.slot_factor, s0.block_map,
                         s0.cache_slots, s0.keys.shape[0] * C8_BLOCK, from_gpu)
        return
    phys = group.states[0].physical_slots(slot_mapping.to(group.device))
    ptrs = torch.tensor(addrs, dtype=torch.int64, device=group.device)
    native().kv_transfer(group.native(), None, ptrs, group.chunk_layout(), 0, 0, chunk_capacity,
                         packets[0].is_cuda, phys, 0, 0, group.num_layers, from_gpu,
                         MODE_AUTO if packets[0].is_cuda else MODE_SIMT, None, None, 0, None)


def indexer_c8_packets_ref(group: IndexerC8GroupState, slot_mapping: torch.Tensor,
                           count: int) -> torch.Tensor:
    """PyTorch oracle: one packet (uint8) for ``count`` tokens from the cache."""
    out = torch.zeros(group.packet_bytes(count), dtype=torch.uint8)
    phys = group.states[0].physical_slots(slot_mapping).cpu()
    row = sum(group.row_bytes)
    for li, s in enumerate(group.states):
        kflat = s.keys.view(-1, 128).view(torch.uint8).view(-1, group.key_bytes).cpu()
        base = li * count * row
        for t in range(count):
            p = int(phys[t])
            if p < 0:
                continue
            out[base + t * group.key_bytes: base + (t + 1) * group.key_bytes] = kflat[p]
            if group.quantized:
                sf = s.scales.view(-1).view(torch.uint8).view(-1, 2).cpu()
                o = base + count * group.key_bytes + t * 2
                out[o:o + 2] = sf[p]
    return out


# ----------------------------------------------------------------- K7
def calculate_cdf(symbols: torch.Tensor, n_bins: int) -> torch.Tensor:
    if symbols.is_cuda:
        return native().calculate_cdf(symbols, n_bins)
    return R.calculate_cdf_ref(symbols, n_bins)


def encode_fast_new(cdf, symbols, output_buffer, output_lengths) -> None:
    if symbols.is_cuda:
        native().encode_fast_new(cdf, symbols, output_buffer, output_lengths)
        return
    out, lens = R.encode_ref(cdf, symbols, output_buffer.shape[2])
    output_buffer.copy_(out)
    output_lengths.copy_(lens)


def decode_fast_prefsum(cdf, bytestreams, lengths, output) -> None:
    if output.is_cuda:
        native().decode_fast_prefsum(cdf, bytestreams, lengths, output)
        return
    output.copy_(R.decode_ref(cdf, bytestreams, lengths, output.shape[1]))


def cachegen_quantize(x: torch.Tensor, bins: torch.Tensor,
                      row_dst: Optional[torch.Tensor] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """x [R, T, C] -> (symbols uint8 [R, T, C], scale fp32 [R, T]); symbol row r
    lands at row ``row_dst[r]``.  half = bins // 2 - 1, scale = max|x| / half,
    q = clamp(round(x / scale) + half, 0, 2 half) per (row, token)."""
    R_, T, C = x.shape
    if x.is_cuda:
        sym = torch.empty(R_, T, C, dtype=torch.uint8, device=x.device)
        scale = torch.empty(R_, T, dtype=torch.float32, device=x.device)
        native().cachegen_quantize(x.contiguous(), bins.to(x.device, torch.int32), sym, scale,
                                   None if row_dst is None
                                   else row_dst.to(x.device, torch.int32))
        return sym, scale
    half = (bins // 2 - 1).view(-1, 1, 1).float()
    amax = x.float().abs().amax(dim=-1, keepdim=True).clamp_min(1e-8)
    sc = amax / half
    q = torch.minimum((torch.round(x.float() / sc) + half).clamp_min(0), 2 * half)
    q = q.to(torch.uint8)
    if row_dst is not None:
        out = torch.empty_like(q)
        out[row_dst.long()] = q
        q = out
    return q, sc.squeeze(-1)


def cachegen_dequantize(sym: torch.Tensor, scale: torch.Tensor, bins: torch.Tensor,
                        dtype: torch.dtype, row_src: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverse of :func:`cachegen_quantize`: y[r] = (sym[row_src[r]] - half) * scale[r]."""
    R_, T = scale.shape
    C = sym.shape[-1]
    if sym.is_cuda:
        y = out if out is not None else torch.empty(R_, T, C, dtype=dtype, device=sym.device)
        native().cachegen_dequantize(sym.contiguous(), scale.contiguous().float(),
                                     bins.to(sym.device, torch.int32), y,
                                     None if row_src is None
                                     else row_src.to(sym.device, torch.int32))
        return y
    src = sym if row_src is None else sym[row_src.long()]
    half = (bins // 2 - 1).view(-1, 1, 1).float()
    y = ((src.float() - half) * scale.float().unsqueeze(-1)).to(dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def decode_fast_new(*args, **kwargs):
    raise NotImplementedError("use decode_fast_prefsum (prefix-summed stream lengths)")


# ----------------------------------------------------------------- K8
def rotary_embedding_k_fused(old_positions, new_positions, key, head_size, cos_sin_cache,
                             is_neox, slot_mapping=None) -> None:
    """Rotate keys in place from ``old_positions`` to ``new_positions``.
    ``slot_mapping`` (optional): token t's row is ``key[slot_mapping[t]]``
    (``key`` a [cache rows, H*D] view of a paged plane; slot -1 skips)."""
    if key.is_cuda:
        native().rotary_embedding_k_fused(old_positions, new_positions, key, head_size,
                                          cos_sin_cache, is_neox, slot_mapping)
        return
    if slot_mapping is None:
        key.copy_(R.rope_delta_ref(old_positions, new_positions, key, head_size,
                                   cos_sin_cache, is_neox).to(key.dtype))
        return
    sm = slot_mapping.long()
    keep = sm >= 0
    rows = key[sm[keep]]
    key[sm[keep]] = R.rope_delta_ref(old_positions[keep], new_positions[keep], rows, head_size,
                                     cos_sin_cache, is_neox).to(key.dtype)


def rotary_embedding_k_fused_layers(old_positions, new_positions, keys, head_size,
                                    cos_sin_cache, is_neox, slot_mapping=None) -> None:
    """The same re-rotation of the key views of several layers (same shape,
    strides and dtype), one launch for all of them on CUDA."""
    if keys and keys[0].is_cuda:
        native().rotary_embedding_k_fused_layers(old_positions, new_positions, list(keys),
                                                 head_size, cos_sin_cache, is_neox,
                                                 slot_mapping)
        return
    for k in keys:
        rotary_embedding_k_fused(old_positions, new_positions, k, head_size, cos_sin_cache,
                                 is_neox, slot_mapping)


# ----------------------------------------------------------------- misc
def layerwise_prefill_dma_copy(dsts: torch.Tensor, srcs: torch.Tensor,
                               sizes: torch.Tensor) -> None:
    native().layerwise_prefill_dma_copy(dsts, srcs, sizes)


def get_gpu_pci_bus_id(device: int = 0) -> str:
    return native().get_gpu_pci_bus_id(device)
