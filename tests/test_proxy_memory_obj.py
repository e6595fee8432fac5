"""Deferred-fetch proxies + transfer contexts: chunks read from a peer's
registered buffer bank by bank and scattered into the paged cache (CPU
tier, TCP channel over loopback ZMQ; the same code drives CUDA connectors)."""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector
from lmcache_ascend_b200.v1.memory_management import MemoryFormat, TensorMemoryAllocator
from lmcache_ascend_b200.v1.proxy_memory_obj import ProxyMemoryObj, load_proxies_pipelined
from lmcache_ascend_b200.v1.transfer_channel.base import BufferConfig
from lmcache_ascend_b200.v1.transfer_channel.tcp_channel import TCPChannel
from lmcache_ascend_b200.v1.transfer_context import P2PTransferContext, PDTransferContext

from .utils import make_separate_kv, random_slots, zeros_like_kv

L, NB, BS, H, D, CS = 2, 32, 16, 2, 32, 64


def _peer_with_chunks(kv, slots, n_tokens):
    """A peer holding the request's chunks, one per page of a host buffer."""
    conn = VLLMPagedMemGPUConnector(LMCacheEngineConfig.from_defaults(chunk_size=CS),
                                    kvcaches=kv)
    shape = conn.get_shape(CS)
    page = shape.numel() * 4
    nchunks = (n_tokens + CS - 1) // CS
    buf = torch.zeros(page * nchunks, dtype=torch.uint8)
    for i in range(nchunks):
        n = min(CS, n_tokens - i * CS)
        view = buf[i * page:i * page + conn.get_shape(n).numel() * 4].view(torch.float32)
        conn.layout.gather_ref(view.view(conn.get_shape(n)), slots[i * CS:i * CS + n])
    ch = TCPChannel("peer", buffers=[BufferConfig(buf, page)])
    return ch, buf, page, shape


@pytest.mark.parametrize("depth", [1, 2, 4])
def test_proxies_resolve_and_scatter_bank_by_bank(depth):
    src = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    T = 5 * CS - 17  # last chunk partial
    s_src = random_slots(T, NB * BS, seed=2)
    peer, buf, page, shape = _peer_with_chunks(src, s_src, T)
    local = TCPChannel("local")
    local.lazy_init_peer_connection("peer", peer.get_local_buffer_refs())
    done = []
    alloc = TensorMemoryAllocator(torch.empty(page * 8, dtype=torch.uint8))
    ctx = PDTransferContext(5, "req-1", done.append, allocator=alloc, shape=shape,
                            dtype=torch.float32, pipeline_depth=depth)
    uuid = next(iter(peer.local))
    starts = [i * CS for i in range(5)]
    ends = [min(T, s + CS) for s in starts]
    dst = zeros_like_kv(src)
    conn = VLLMPagedMemGPUConnector(LMCacheEngineConfig.from_defaults(chunk_size=CS),
                                    kvcaches=dst)
    proxies = [ProxyMemoryObj(conn.get_shape(e - s), torch.float32, MemoryFormat.KV_2LTD, local,
                              "peer", (uuid, i), ctx) for i, (s, e) in enumerate(zip(starts, ends))]
    s_dst = random_slots(T, NB * BS, seed=3)
    try:
        conn.batched_to_gpu(proxies, starts, ends, slot_mapping=s_dst)
        for l in range(L):
            for p in range(2):
                a = src[l][p].reshape(NB * BS, -1)[s_src]
                b = dst[l][p].reshape(NB * BS, -1)[s_dst]
                assert torch.equal(a, b)
        assert done == ["req-1"] and all(p.consumed for p in proxies)
        assert alloc.num_active == 0 and alloc.memcheck()
    finally:
        local.close()
        peer.close()


def test_context_done_once_early_and_buffer_accounting():
    sent = []
    alloc = TensorMemoryAllocator(torch.empty(4096, dtype=torch.uint8))
    ctx = P2PTransferContext(3, "lk", "tcp://peer", lambda peer, lid: sent.append((peer, lid)),
                             allocator=alloc, shape=torch.Size([256]), dtype=torch.float32,
                             pipeline_depth=8)
    assert ctx.max_pipeline_depth == 3  # capped by the number of proxies
    bufs = ctx.allocate_buffers(3)
    with pytest.raises(MemoryError):
        ctx.allocate_buffers(2)  # 3 KiB of 4 KiB used: all-or-none
    assert alloc.num_active == 3
    ctx.decref()
    ctx.send_done_now()  # retrieve gave up early
    ctx.decref()
    ctx.decref()  # last proxy: Done already sent, not resent
    assert sent == [("tcp://peer", "lk")]
    ctx.release_buffers(bufs[:1])
    ctx.close()  # releases the rest
    assert alloc.num_active == 0 and alloc.memcheck()


def test_pipeline_waits_for_bank_scatter_before_refill():
    order = []

    class Ev:
        def __init__(self, k):
            self.k = k

        def synchronize(self):
            order.append(("wait_scatter", self.k))

    class Chan:
        def submit_batched_read(self, dsts, peer, addrs):
            order.append(("read", [a[1] for a in addrs]))
            return None

    alloc = TensorMemoryAllocator(torch.empty(1 << 16, dtype=torch.uint8))
    ctx = PDTransferContext(6, "r", lambda _: None, allocator=alloc, shape=torch.Size([16]),
                            dtype=torch.float32, pipeline_depth=4)
    ch = Chan()
    px = [ProxyMemoryObj(torch.Size([16]), torch.float32, MemoryFormat.KV_2LTD, ch, "p",
                         ("u", i), ctx) for i in range(6)]
    k = [0]

    def scatter(objs, s, e):
        order.append(("scatter", [o.remote_addr[1] for o in objs]))
        k[0] += 1
        return Ev(k[0])

    load_proxies_pipelined(px, list(range(6)), list(range(1, 7)), scatter)
    # banks of 2: read b0, read b1 (overlaps scatter b0), wait scatter b0 before refilling it
    assert order[:4] == [("read", [0, 1]), ("read", [2, 3]), ("scatter", [0, 1]),
                         ("wait_scatter", 1)]
    assert ("read", [4, 5]) in order and order.index(("read", [4, 5])) > 3
    assert alloc.num_active == 0
