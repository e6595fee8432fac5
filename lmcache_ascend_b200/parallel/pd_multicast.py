"""PD push fan-out through NVSwitch multicast (NVLS).

One prefiller sends the same KV to several decoders (a TP-replicated MLA
latent cache, or a decoder group larger than the prefill group) while its
NVLink egress carries the bytes once: the group's members share a symmetric
staging buffer bound to an NVLink multicast object
(``torch.distributed._symmetric_memory``), the prefiller's kernel stores every
vector once with ``multimem.st`` and bumps per-layer flags with
``multimem.red.release``, and each decoder waits on its own copy of the flags
(bounded) and scatters the staging rows into its paged cache locally.

Construction is collective over ``group`` (every member passes the same
shapes).  ``has_multicast`` is False where the system has no NVLS; callers
then use ``PushSender`` fan-out (one peer store per decoder).

Reuse of the one staging buffer: every member other than the pushing member
(``root``) hands each push back when it is done with it -- ``scatter`` does so
when its layer range ends at the last layer, or call ``release`` -- by adding
1 to a counter in the root's buffer (a peer atomic, not a multicast store).
Push k (from 0) first waits, on the root's stream and bounded, until that
counter has reached k * (members - 1), so a push never overwrites rows a
member is still scattering.  A wait that runs out reports a flag timeout in
``status`` and the push's rows are then not to be trusted.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from ..v1.kv_format import PagedKVLayout


class MulticastFanout:
    def __init__(self, group, num_layers: int, num_planes: int, row_bytes: int,
                 max_tokens: int, device: torch.device, root: int = 0):
        import torch.distributed._symmetric_memory as symm_mem

        self.num_layers, self.num_planes = num_layers, num_planes
        self.row_bytes, self.max_tokens = row_bytes, max_tokens
        self.device = torch.device(device)
        self.root = root
        rows = num_layers * num_planes * max_tokens * row_bytes
        self.flags_off = (rows + 255) // 256 * 256
        self.release_off = self.flags_off + 4 * max(num_layers, 1)  # root's release counter
        self.buf = symm_mem.empty(self.release_off + 16, dtype=torch.uint8,
                                  device=self.device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group)
        from torch._C._autograd import DeviceType

        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.has_multicast = bool(
            symm_mem._SymmetricMemory.has_multicast_support(DeviceType.CUDA, idx))
        self.mc = self._multicast_addr() if self.has_multicast else 0
        self.has_multicast = self.mc != 0
        self.members = int(self.handle.world_size)
        self.is_root = int(self.handle.rank) == root
        # the root's release counter, as this process addresses it
        mine = int(self.handle.buffer_ptrs[self.handle.rank])
        self._root_counter = (int(self.handle.buffer_ptrs[root]) + (self.buf.data_ptr() - mine)
                              + self.release_off)
        self._pushes = 0
        torch.cuda.synchronize(self.device)
        # zeroed flags visible to every member before any push (bounded wait)
        self.handle.barrier(0, 30000)
        self.expected = [0] * num_layers
        self.status = ops.DeviceStatus(self.device)
        # row ((layer * planes + p) * T + t): plane p starts p * rb * T in,
        # layer l at l * planes * rb * T, token t at t * rb
        rb, npl = row_bytes, num_planes
        self._chunk_layout = ops.native().ChunkLayout([rb] * npl, npl * rb, [rb] * npl,
                                                      [0] * npl)

    def _multicast_addr(self) -> int:
        """Multicast address of ``self.buf``'s first byte, or 0 when the
        tensor cannot be located inside the handle's allocation (multicast is
        then left off rather than storing at an unverified address)."""
        mc = int(self.handle.multicast_ptr)
        if mc == 0:
            return 0
        base = int(self.handle.buffer_ptrs[self.handle.rank])
        off = int(getattr(self.handle, "offset", 0) or 0)
        data = self.buf.data_ptr()
        if data == base + off:
            return mc + off
        if data == base and off == 0:
            return mc
        return 0

    # ------------------------------------------------------------ sender
    def push(self, layout: PagedKVLayout, src_slots: torch.Tensor, tile_tokens: int = 128,
             grid: int = 0, release_timeout_s: float = 10.0) -> None:
        """Root only: enqueue the push of every layer on the current stream,
        after a bounded wait until every other member released the previous
        push."""
        if not self.has_multicast:
            raise RuntimeError("NVLink multicast is not available on this system")
        if not self.is_root:
            raise RuntimeError("only the root member pushes")
        if src_slots.numel() > self.max_tokens:
            raise ValueError("push larger than the multicast staging area")
        if self._pushes > 0 and self.members > 1:
            target = (self._pushes * (self.members - 1)) & 0xFFFFFFFF
            ops.native().pd_wait_value(self.buf.data_ptr() + self.release_off, target,
                                       release_timeout_s, self.status.tensor)
        self._pushes += 1
        ops.native().pd_push_multimem(layout.native(), self.mc, self.mc + self.flags_off,
                                      src_slots, 0, self.num_layers, tile_tokens, grid,
                                      self.status.tensor)

    # ---------------------------------------------------------- receiver
    def expect(self, num_tokens: int, tile_tokens: int = 128) -> torch.Tensor:
        units = ops.native().push_units_per_layer(num_tokens, self.num_planes, tile_tokens)
        tg = []
        for l in range(self.num_layers):
            self.expected[l] = (self.expected[l] + units) & 0xFFFFFFFF
            tg.append(self.expected[l] - (1 << 32) if self.expected[l] >= (1 << 31)
                      else self.expected[l])
        return torch.tensor(tg, dtype=torch.int32).to(self.device, non_blocking=True)

    def wait(self, targets: torch.Tensor, timeout_s: float = 10.0, layer_begin: int = 0) -> None:
        """Bounded device wait until layers ``layer_begin ..`` (one target
        each, from ``expect``) have landed in this member's staging."""
        ops.native().pd_wait_flags(self.buf.data_ptr() + self.flags_off, targets, layer_begin,
                                   timeout_s, self.status.tensor)

    def scatter(self, layout: PagedKVLayout, dst_slots: torch.Tensor, num_tokens: int,
                layer_begin: int = 0, num_layers: Optional[int] = None,
                release: Optional[bool] = None) -> None:
        """Local staging rows of the last push -> this member's paged cache
        (layers ``layer_begin .. layer_begin + num_layers``).  ``release``
        (default: when the range ends at the last layer, on a member other
        than the root) hands the staging back to the root afterwards."""
        n = self.num_layers - layer_begin if num_layers is None else num_layers
        ops.native().kv_transfer(layout.native(), self.buf, None, self._chunk_layout,
                                 num_tokens, 0, 0, True, dst_slots, layer_begin, layer_begin, n,
                                 False, 0, self.status.tensor, None, 0, None)
        if release is None:
            release = not self.is_root and layer_begin + n >= self.num_layers
        if release:
            self.release()

    def release(self) -> None:
        """Member other than the root: hand the last push's staging back to
        the root (stream-ordered after the work enqueued so far)."""
        if self.is_root:
            return
        ops.native().pd_flag_add(self._root_counter, 1)

    def check(self) -> None:
        self.status.check("multicast fan-out")
