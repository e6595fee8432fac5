"""Disaggregated-prefill KV push over NVLink (host side of the K9 kernel).

Roles:
* ``PushReceiver`` (decoder rank): describes its paged KV cache and a small
  flag array (one cumulative counter per layer, in its own HBM) as CUDA IPC
  descriptors, and waits for pushed layers with a bounded device-side spin.
* ``PushSender`` (prefiller rank): maps the receiver's planes and flags into
  its address space and launches ``pd_push``: one kernel that reads the
  prefiller's paged rows and stores them into the decoder's paged blocks
  through peer addresses (NVLink / NVSwitch), then releases each layer's flag.

The exchange of descriptors is left to the caller (torch.distributed object
collectives in the benchmark, the PD backend's ZMQ handshake in serving).
Fan-out to several receivers (TP-replicated MLA latent) is one launch with
``replicas`` destination tables; the rows are read once.

Optional block-scaled fp8 transfer (``quant="fp8"``): the same kernel pass
quantises each group of 128 bf16 elements to e4m3 with one fp32 scale and
stores them into a staging area in the receiver's HBM, so about half the
bytes cross NVLink; the receiver dequantises into its bf16 paged cache after
the layer flags (``PushReceiver.dequantize``).  Lossy: the relative error of
an element is at most 2^-4 of its group's maximum.

The staging area holds ``fp8_buffers`` requests (two by default), used in
turn.  A push whose ``layer_begin`` is 0 starts a new request in the next
buffer; before it writes into a buffer that an earlier request used, the
sender's stream waits (bounded, on the device) until the receiver has released
that request.  The receiver releases a request when it dequantises the last
layer (or when ``dequantize(..., release=True)``) by adding 1 to a counter in
its own HBM.  A wait that runs out reports a flag timeout through the sender's
status, and the staging contents are then not to be trusted.
"""

from __future__ import annotations

import uuid
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops
from ..v1.kv_format import PagedKVLayout
from .ipc import IpcDesc, PeerMappings, export_local

# tokens per flag unit (one release per (layer, plane, tile)); sender and
# receiver must use the same value for a push
PUSH_TILE = 512


@dataclass
class ReceiverDesc:
    num_layers: int
    block_size: int
    num_slots: int
    block_stride: List[int]
    slot_stride: List[int]
    row_bytes: List[int]
    planes: List[List[dict]]  # [layer][plane] -> IpcDesc dict
    flags: dict               # IpcDesc dict of the flag array
    device: int
    seg_bytes: List[int] = field(default_factory=list)   # head-major rows (0: contiguous)
    seg_stride: List[int] = field(default_factory=list)
    fp8_q: Optional[dict] = None        # IpcDesc dict of the fp8 staging rows
    fp8_scales: Optional[dict] = None   # IpcDesc dict of the staging scales
    fp8_tokens: int = 0                 # staging capacity in tokens per push
    fp8_group: int = 128
    fp8_buffers: int = 1                # requests the staging holds at once
    fp8_q_stride: int = 0               # bytes between staging buffers (rows)
    fp8_s_stride: int = 0               # bytes between staging buffers (scales)
    fp8_release_index: int = -1         # flag word the receiver bumps per released request
    # registration epoch: a new one per PushReceiver, so a sender holding a
    # mapping of an earlier registration (re-allocated or restarted decoder)
    # is refused before it writes
    epoch: str = ""

    def to_dict(self) -> dict:
        return self.__dict__.copy()

    @staticmethod
    def from_dict(d: dict) -> "ReceiverDesc":
        return ReceiverDesc(**d)


class PushReceiver:
    def __init__(self, layout: PagedKVLayout, max_layers: Optional[int] = None,
                 fp8_staging_tokens: int = 0, fp8_group: int = 128, fp8_buffers: int = 2):
        self.layout = layout
        self.device = layout.device
        dev = self.device.index or 0
        n = max(layout.num_layers, max_layers or 0)
        self._release_index = max(n, 1)  # one word after the layer flags
        self._flags_buf = ops.native().device_buffer(4 * (self._release_index + 1), dev)
        self.flags = self._flags_buf.view(torch.int32)
        self.expected = [0] * n  # cumulative flag target per layer
        self.status = ops.DeviceStatus(self.device)
        planes = []
        for layer in range(layout.num_layers):
            row = []
            for p in layout.planes:
                row.append(export_local(p.views[layer].data_ptr(), dev).to_dict())
            planes.append(row)
        es = layout.elem_size
        self.desc = ReceiverDesc(
            num_layers=layout.num_layers, block_size=layout.block_size,
            num_slots=layout.num_slots,
            block_stride=[p.views[0].stride(0) * es for p in layout.planes],
            slot_stride=[p.views[0].stride(1) * es for p in layout.planes],
            row_bytes=layout.row_bytes, planes=planes,
            flags=export_local(self._flags_buf.data_ptr(), dev).to_dict(), device=dev,
            seg_bytes=[p.seg_elems * es if p.segmented else 0 for p in layout.planes],
            seg_stride=[p.seg_stride * es if p.segmented else 0 for p in layout.planes],
            epoch=uuid.uuid4().hex)
        self.fp8_tokens, self.fp8_group = fp8_staging_tokens, fp8_group
        if fp8_staging_tokens > 0:
            mod = ops.native()
            nat = layout.native()
            qb = mod.fp8_staging_bytes(nat, fp8_staging_tokens, layout.num_layers, fp8_group,
                                       False)
            sb = mod.fp8_staging_bytes(nat, fp8_staging_tokens, layout.num_layers, fp8_group,
                                       True)
            if fp8_buffers < 1:
                raise ValueError("fp8_buffers must be >= 1")
            sb = (sb + 15) // 16 * 16
            self._fp8_nb, self._fp8_qb, self._fp8_sb = fp8_buffers, qb, sb
            self._q_buf = mod.device_buffer(qb * fp8_buffers, dev)
            self._s_buf = mod.device_buffer(sb * fp8_buffers, dev)
            self._fp8_seq = 0  # next request to dequantise
            self.desc.fp8_q = export_local(self._q_buf.data_ptr(), dev).to_dict()
            self.desc.fp8_scales = export_local(self._s_buf.data_ptr(), dev).to_dict()
            self.desc.fp8_tokens = fp8_staging_tokens
            self.desc.fp8_group = fp8_group
            self.desc.fp8_buffers = fp8_buffers
            self.desc.fp8_q_stride, self.desc.fp8_s_stride = qb, sb
            self.desc.fp8_release_index = self._release_index

    def expect_host(self, num_tokens: int, layer_begin: int = 0,
                    num_layers: Optional[int] = None,
                    tile_tokens: int = PUSH_TILE) -> List[int]:
        """Record one incoming push; returns the per-layer flag targets (host
        list; any thread may call this, nothing touches the device)."""
        nl = self.layout.num_layers - layer_begin if num_layers is None else num_layers
        units = ops.native().push_units_per_layer(num_tokens, self.layout.num_planes,
                                                  tile_tokens)
        tg = []
        for l in range(layer_begin, layer_begin + nl):
            self.expected[l] = (self.expected[l] + units) & 0xFFFFFFFF
            tg.append(self.expected[l] - (1 << 32) if self.expected[l] >= (1 << 31)
                      else self.expected[l])
        return tg

    def expect(self, num_tokens: int, layer_begin: int = 0,
               num_layers: Optional[int] = None, tile_tokens: int = PUSH_TILE) -> torch.Tensor:
        """Record one incoming push; returns the device targets for ``wait``."""
        tg = self.expect_host(num_tokens, layer_begin, num_layers, tile_tokens)
        return torch.tensor(tg, dtype=torch.int32).to(self.device, non_blocking=True)

    def wait(self, targets, layer_begin: int = 0, timeout_s: float = 10.0) -> None:
        """Enqueue a bounded wait on the current stream (no host sync).
        ``targets``: device tensor from ``expect``, or the host list of
        ``expect_host`` (copied from pinned memory on the current stream)."""
        if not isinstance(targets, torch.Tensor):
            host = torch.tensor(targets, dtype=torch.int32).pin_memory()
            targets = host.to(self.device, non_blocking=True)
        ops.native().pd_wait_flags(self._flags_buf.data_ptr(), targets, layer_begin,
                                   timeout_s, self.status.tensor)

    def dequantize(self, dst_slots: torch.Tensor, layer_begin: int = 0,
                   num_layers: Optional[int] = None, release: Optional[bool] = None) -> None:
        """After ``wait``: fp8 staging of the current request -> bf16 paged
        cache at ``dst_slots`` (enqueued on the current stream).  ``release``
        (default: when the range ends at the last layer) hands the request's
        staging buffer back to the sender after this dequantisation."""
        if self.fp8_tokens <= 0:
            raise RuntimeError("receiver was built without fp8 staging")
        if dst_slots.numel() > self.fp8_tokens:
            raise ValueError("push larger than the fp8 staging area")
        nl = self.layout.num_layers - layer_begin if num_layers is None else num_layers
        b = self._fp8_seq % self._fp8_nb
        ops.native().pd_dequant_scatter(self.layout.native(),
                                        self._q_buf.data_ptr() + b * self._fp8_qb,
                                        self._s_buf.data_ptr() + b * self._fp8_sb, dst_slots,
                                        layer_begin, nl, self.fp8_group, self.status.tensor)
        if release is None:
            release = layer_begin + nl >= self.layout.num_layers
        if release:
            self.release_staging()

    def release_staging(self) -> None:
        """Hand the current request's fp8 staging buffer back to the sender
        (stream-ordered after the work already enqueued)."""
        ops.native().pd_flag_add(self._flags_buf.data_ptr() + 4 * self._release_index, 1)
        self._fp8_seq += 1

    def check(self) -> None:
        self.status.check("pd push receiver")


_ENGINES = {"auto": 0, "bulk": 1, "simt": 2}


class PushSender:
    """``engine`` picks the kernel of the lossless push; every engine releases
    the same per-layer flags, and the decoder may be on this GPU (loopback)
    or on a peer GPU (NVLink), with the same kernel either way:

    * "bulk": TMA bulk copies (`cp.async.bulk`, non-multicast) through a
      shared-memory ring, runs of contiguous rows merged into one copy;
      needs 16-byte aligned, contiguous (token-major) rows on both sides;
    * "simt": 16-byte vector loads and stores per lane; any row layout,
      including head-major segmented rows;
    * "auto" (default): through a peer mapping (the decoder on another GPU)
      "simt", which moved 703.8 GB/s per pair against 688.8 for "bulk" on
      the same B200 pair; on this GPU "bulk" when both layouts allow it
      (0.79 against 0.64 of HBM for "simt"), else "simt".
    """

    def __init__(self, layout: PagedKVLayout, engine: str = "auto"):
        if engine not in _ENGINES:
            raise ValueError(f"engine must be one of {sorted(_ENGINES)}")
        self.engine = engine
        self.layout = layout
        self.device = layout.device
        self.peers = PeerMappings(self.device.index or 0)
        self.status = ops.DeviceStatus(self.device)
        self._dst = None
        self._flag_ptrs: List[int] = []
        self.replicas = 0
        self._last_push: Optional[torch.cuda.Event] = None  # unmap only after it
        # per-unit completion counters of the bulk engine (zero between
        # launches; launches of one sender run in stream order)
        self._counters: Optional[torch.Tensor] = None
        self._old_counters: List[torch.Tensor] = []

    def connect(self, receivers: Sequence[ReceiverDesc]) -> None:
        """Map one or more receivers (same layout, fan-out) for pushing."""
        mod = ops.native()
        r0 = receivers[0]
        for r in receivers:
            if (r.row_bytes != self.layout.row_bytes or r.num_layers != r0.num_layers
                    or r.block_size != r0.block_size or r.block_stride != r0.block_stride
                    or r.slot_stride != r0.slot_stride or r.seg_bytes != r0.seg_bytes
                    or r.seg_stride != r0.seg_stride):
                raise ValueError("receiver layouts must match the sender's rows and each other")
        ptrs = []
        for r in receivers:
            for layer in range(r.num_layers):
                for pd in r.planes[layer]:
                    ptrs.append(self.peers.resolve(IpcDesc.from_dict(pd)))
        table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self._dst = mod.PagedLayout(table, r0.block_stride, r0.slot_stride, r0.row_bytes,
                                    r0.block_size, r0.num_slots, list(r0.seg_bytes),
                                    list(r0.seg_stride))
        self._dst.set_bases_aligned(all(p % 16 == 0 for p in ptrs))
        self._flag_ptrs = [self.peers.resolve(IpcDesc.from_dict(r.flags)) for r in receivers]
        self.replicas = len(receivers)
        try:
            here = mod.get_gpu_pci_bus_id(self.device.index or 0)
        except Exception:  # pragma: no cover - no bus id: treat as local
            here = ""
        buses = [IpcDesc.from_dict(r.flags).pci_bus_id for r in receivers]
        self._remote = bool(here) and any(b not in ("", here) for b in buses)
        # flags released at GPU scope only when every receiver is known to be
        # on this GPU (an unknown bus id keeps system scope)
        self._all_local = bool(here) and all(b == here for b in buses)
        self._fp8 = None
        self._fp8_seq, self._fp8_buf = 0, 0
        if r0.fp8_q is not None and len(receivers) == 1:
            rel = (self._flag_ptrs[0] + 4 * r0.fp8_release_index
                   if r0.fp8_release_index >= 0 else 0)
            self._fp8 = (self.peers.resolve(IpcDesc.from_dict(r0.fp8_q)),
                         self.peers.resolve(IpcDesc.from_dict(r0.fp8_scales)),
                         r0.fp8_tokens, r0.fp8_group, max(1, r0.fp8_buffers),
                         r0.fp8_q_stride, r0.fp8_s_stride, rel)

    def push(self, src_slots: torch.Tensor, dst_slots: torch.Tensor, layer_begin: int = 0,
             num_layers: Optional[int] = None, tile_tokens: int = PUSH_TILE, grid: int = 0,
             quant: str = "none", staging_timeout_s: float = 10.0) -> None:
        """Enqueue the push of ``num_layers`` layers on the current stream.
        ``quant="fp8"`` sends block-scaled fp8 to the receiver's staging (the
        receiver applies ``dst_slots`` in ``PushReceiver.dequantize``); a push
        from layer 0 starts a new request in the next staging buffer, after a
        bounded device wait (``staging_timeout_s``) for the receiver to have
        released that buffer's previous request."""
        if self._dst is None:
            raise RuntimeError("PushSender.connect() first")
        nl = self.layout.num_layers - layer_begin if num_layers is None else num_layers
        if quant == "fp8":
            if self._fp8 is None:
                raise RuntimeError("fp8 push needs one receiver built with fp8 staging")
            q_ptr, s_ptr, cap, group, nb, qst, sst, rel = self._fp8
            if src_slots.numel() > cap:
                raise ValueError("push larger than the receiver's fp8 staging area")
            if layer_begin == 0 or self._fp8_seq == 0:
                seq = self._fp8_seq
                self._fp8_seq += 1
                self._fp8_buf = seq % nb
                if seq >= nb and rel:
                    ops.native().pd_wait_value(rel, seq - nb + 1, staging_timeout_s,
                                               self.status.tensor)
            b = self._fp8_buf
            ops.native().pd_push_fp8(self.layout.native(), q_ptr + b * qst, s_ptr + b * sst,
                                     src_slots, layer_begin, nl, self._flag_ptrs[0],
                                     tile_tokens, grid, group, self.status.tensor,
                                     getattr(self, "_all_local", False))
            self._mark_pushed()
            return
        if quant != "none":
            raise ValueError("quant must be 'none' or 'fp8'")
        units = ops.native().push_units_per_layer(src_slots.numel(), self.layout.num_planes,
                                                  tile_tokens) * nl
        if self._counters is None or self._counters.numel() < units:
            if self._counters is not None:  # an earlier launch may still use it
                self._old_counters.append(self._counters)
            self._counters = torch.zeros(max(units, 1 << 16), dtype=torch.int32,
                                         device=self.device)
        ops.native().pd_push(self.layout.native(), self._dst, src_slots, dst_slots,
                             layer_begin, nl, self.replicas, self._flag_ptrs, tile_tokens,
                             grid, self.status.tensor, self._mode(), self._counters,
                             getattr(self, "_all_local", False))
        self._mark_pushed()

    def _mode(self) -> int:
        if self.engine == "auto" and getattr(self, "_remote", False):
            return _ENGINES["simt"]
        return _ENGINES[self.engine]

    def _mark_pushed(self) -> None:
        if self._last_push is None:
            self._last_push = torch.cuda.Event()
        self._last_push.record()

    def check(self) -> None:
        try:
            self.status.check("pd push sender")
        except RuntimeError:
            # a push that stopped early leaves unit counters half counted
            if self._counters is not None:
                self._counters.zero_()
            raise

    def close(self) -> None:
        """Unmap the receivers, after the pushes enqueued so far have run
        (the event is recorded on whichever stream launched the last push)."""
        if self._last_push is not None:
            self._last_push.synchronize()
        self.peers.close()
        self._dst = None
        self.replicas = 0
