"""PD (disaggregated prefill) control-plane messages.

msgspec structs exchanged over ZMQ between the sender (prefiller) and the
receiver (decoder).  Names and fields follow the protocol the reference
speaks (AllocRequest / AllocResponse / ProxyNotif from upstream LMCache's
pd_backend, extended in reference lmcache_ascend/v1/storage_backend/pd/
messages.py:21-86 with buffer UUIDs, alloc_failed and the pull-mode
messages).  Added here: the channel handshake and the direct paged push
(prefiller paged blocks -> decoder paged blocks, no chunk buffers).
"""

from __future__ import annotations

from typing import List, Optional, Union

import msgspec


class AllocRequest(msgspec.Struct, tag=True):
    keys: List[str]
    fmt: int
    shape: List[int]
    dtype: str
    last_chunk_toks: int
    sender_id: str = ""


class AllocResponse(msgspec.Struct, tag=True):
    already_sent_indexes: List[int]
    remote_indexes: List[int]
    remote_buffer_uuids: List[str] = []
    alloc_failed: bool = False


class ProxyNotif(msgspec.Struct, tag=True):
    req_id: str


class PullReadyNotif(msgspec.Struct, tag=True):
    pull_id: str
    keys: List[str]
    sender_buffer_uuids: List[str]
    sender_mem_indexes: List[int]
    sender_id: str
    sender_done_url: str
    fmt: int
    shape: List[int]
    dtype: str
    last_chunk_toks: int


class PullReadyDoneAck(msgspec.Struct, tag=True):
    already_sent_indexes: List[int]
    alloc_failed: bool = False


class PullDoneSignal(msgspec.Struct, tag=True):
    pull_id: str


class HandshakeRequest(msgspec.Struct, tag=True):
    """Channel set-up: the peer's registered buffers (and, for the direct
    push, its paged-KV receiver descriptor)."""

    peer_id: str
    buffer_refs: List[dict]
    receiver_desc: Optional[dict] = None


class HandshakeResponse(msgspec.Struct, tag=True):
    peer_id: str
    buffer_refs: List[dict]
    receiver_desc: Optional[dict] = None
    ok: bool = True
    error: str = ""


class DirectPushNotif(msgspec.Struct, tag=True):
    """Sent by the prefiller after enqueuing a direct paged push, so the
    decoder knows how many flag units each layer will receive."""

    req_id: str
    num_tokens: int
    layer_begin: int
    num_layers: int
    tile_tokens: int
    keys: List[str] = []


class WriteDone(msgspec.Struct, tag=True):
    """Sent by the sender once the pages for ``keys`` have been written;
    the receiver only reports them as present after this."""

    keys: List[str]


class Ack(msgspec.Struct, tag=True):
    ok: bool = True
    error: str = ""


PDMsg = Union[AllocRequest, AllocResponse, ProxyNotif, PullReadyNotif, PullReadyDoneAck,
              PullDoneSignal, HandshakeRequest, HandshakeResponse, DirectPushNotif, WriteDone,
              Ack]

_enc = msgspec.msgpack.Encoder()
_dec = msgspec.msgpack.Decoder(PDMsg)


def encode(msg) -> bytes:
    return _enc.encode(msg)


def decode(data: bytes):
    return _dec.decode(data)
