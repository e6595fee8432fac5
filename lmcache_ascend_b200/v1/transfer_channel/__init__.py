"""Transfer channels (factory mirrors reference
lmcache_ascend/v1/transfer_channel/__init__.py:95-170).

``nvlink`` replaces the reference's hccl / hixl / hcomm_onesided channels on
one B200 box; ``tcp`` moves host buffers over ZMQ (CPU tier, cross-box)."""

from __future__ import annotations

from typing import Optional

from .base import BaseTransferChannel, BufferConfig, RemoteAddr


def CreateTransferChannel(channel_type: str, peer_id: str, buffers=None,
                          device=None, endpoint: Optional[str] = None,
                          **kw) -> BaseTransferChannel:
    t = {"hccl": "nvlink", "hixl": "nvlink", "hcomm_onesided": "nvlink",
         "nixl": "nvlink"}.get(channel_type, channel_type)
    if t == "nvlink":
        from .nvlink_channel import NVLinkChannel

        return NVLinkChannel(peer_id, device=device, buffers=buffers)
    if t == "tcp":
        from .tcp_channel import TCPChannel

        return TCPChannel(peer_id, endpoint=endpoint or "tcp://127.0.0.1:*", buffers=buffers,
                          **kw)
    raise ValueError(f"unknown transfer channel {channel_type!r}")


__all__ = ["BaseTransferChannel", "BufferConfig", "CreateTransferChannel", "RemoteAddr"]
