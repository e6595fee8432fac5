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


class DirectPushReserve(msgspec.Struct, tag=True):
    """Sent by the prefiller BEFORE it launches any kernel that stores into
    the decoder's paged blocks.  The decoder grants it only if ``epoch`` is
    its current registration (its cache has not been re-registered or
    re-allocated since the sender mapped it), every destination slot is in
    range, and -- unless the decoder runs without reservations -- the
    destination slots are exactly the ones the decoder reserved for
    ``req_id`` (compared by digest).  The grant also tells the decoder how
    many flag units each layer will receive."""

    req_id: str
    epoch: str
    num_tokens: int        # tokens of this push (-1 with want_slots: as many as reserved)
    layer_begin: int
    num_layers: int
    tile_tokens: int
    dst_digest: str        # digest of the sender's destination slots ("" with want_slots)
    dst_max_slot: int
    sender_id: str = ""
    token_begin: int = 0   # first token of the reservation this push covers
    want_slots: bool = False  # the sender has no slots: the grant carries the reserved ones
    prompt_end: int = -1   # with want_slots: the sender holds KV of prompt positions < this


class DirectPushGrant(msgspec.Struct, tag=True):
    ok: bool
    epoch: str = ""
    error: str = ""
    retry: bool = False  # refused for now (no reservation yet); asking again may succeed
    slots: List[int] = []  # with want_slots: the granted destination slots
    first_token: int = 0   # prompt position of the reservation's first token


class WriteDone(msgspec.Struct, tag=True):
    """Sent by the sender once the pages for ``keys`` have been written;
    the receiver only reports them as present after this."""

    keys: List[str]


class Ack(msgspec.Struct, tag=True):
    ok: bool = True
    error: str = ""


PDMsg = Union[AllocRequest, AllocResponse, ProxyNotif, PullReadyNotif, PullReadyDoneAck,
              PullDoneSignal, HandshakeRequest, HandshakeResponse, DirectPushReserve,
              DirectPushGrant, WriteDone, Ack]

_enc = msgspec.msgpack.Encoder()
_dec = msgspec.msgpack.Decoder(PDMsg)


def encode(msg) -> bytes:
    return _enc.encode(msg)


def decode(data: bytes):
    return _dec.decode(data)


def slot_digest(slots) -> "tuple[str, int]":
    """(digest, max slot) of a destination slot list (host tensor or
    sequence).  Both sides of a direct push compute it over the same int64
    little-endian bytes."""
    import zlib

    import numpy as np
    import torch

    if isinstance(slots, torch.Tensor):
        arr = slots.detach().to("cpu", torch.int64).numpy()
    elif isinstance(slots, np.ndarray):
        arr = slots
    else:
        arr = np.asarray(list(slots), dtype=np.int64)
    a64 = np.ascontiguousarray(arr.astype("<i8", copy=False))
    # a consistency check (both ends are trusted): CRC-32 of the bytes, the
    # element sum and the length
    h = f"{zlib.crc32(memoryview(a64)):08x}{int(a64.sum()) & 0xFFFFFFFFFFFF:012x}{a64.size:x}"
    return h, int(a64.max()) if a64.size else -1
