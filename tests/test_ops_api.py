"""Reference-named op surface (ops/api.py): single-layer, sparse, flash
layout, multi-chunk direct, CUDA-graph sparse copy and the C8 indexer
transfer; CPU oracle paths and CUDA kernels compared bit-exact."""

import pytest
import torch

from lmcache_ascend_b200.ops import api
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

from .utils import block_slots, make_separate_kv, random_slots

GPU = pytest.mark.gpu


def _devs():
    return ["cpu", pytest.param("cuda", marks=GPU)]


@pytest.mark.parametrize("dev", _devs())
@pytest.mark.parametrize("token_major", [False, True])
def test_single_layer_round_trip(dev, token_major):
    kv = make_separate_kv(3, 32, 16, 4, 64, torch.bfloat16, dev, seed=1)
    lay = PagedKVLayout(kv)
    T = 100
    slots = random_slots(T, 512, seed=2, device=dev)
    shape = (T, 2, 256) if token_major else (2, T, 256)
    buf = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
    api.single_layer_kv_transfer(buf, lay, 1, slots, True, token_major)
    k, v = kv[1]
    want_k = k.reshape(-1, 256)[slots.long()]
    got_k = buf[:, 0] if token_major else buf[0]
    assert torch.equal(got_k, want_k)
    kv2 = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in kv]
    lay2 = PagedKVLayout(kv2)
    api.single_layer_kv_transfer(buf, lay2, 1, slots, False, token_major)
    assert torch.equal(kv2[1][1].reshape(-1, 256)[slots.long()], v.reshape(-1, 256)[slots.long()])


@pytest.mark.parametrize("dev", _devs())
def test_sparse_single_layer(dev):
    kv = make_separate_kv(2, 32, 16, 4, 64, torch.float16, dev, seed=3)
    kv2 = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in kv]
    lay2 = PagedKVLayout(kv2)
    T = 128
    staging = torch.randn(2, T, 256, device=dev).to(torch.float16)
    sel = torch.randperm(T, device=dev)[:40]
    slots = random_slots(40, 512, seed=4, device=dev)
    api.sparse_single_layer_kv_transfer(staging, lay2, 0, slots, sel)
    k2 = kv2[0][0].reshape(-1, 256)
    assert torch.equal(k2[slots.long()], staging[0][sel.long()])


@pytest.mark.parametrize("dev", _devs())
def test_flash_layout_layer(dev):
    kv = make_separate_kv(4, 32, 16, 2, 64, torch.bfloat16, dev, seed=5)
    lay = PagedKVLayout(kv)
    T = 64
    slots = block_slots(T, 16, 32, seed=6, device=dev)
    buf = torch.zeros(lay.chunk_shape(T), dtype=torch.bfloat16, device=dev)
    api.reshape_and_cache_back_flash(buf, lay, 2, slots)
    assert torch.equal(buf[0, 2], kv[2][0].reshape(-1, 128)[slots.long()])
    assert int(buf[:, 0].abs().sum()) == 0  # other layers untouched
    kv2 = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in kv]
    lay2 = PagedKVLayout(kv2)
    api.load_and_reshape_flash(buf, lay2, 2, slots)
    assert torch.equal(kv2[2][1].reshape(-1, 128)[slots.long()], buf[1, 2])


@pytest.mark.parametrize("dev", _devs())
def test_direct_multi_chunk(dev):
    kv = make_separate_kv(2, 64, 16, 2, 64, torch.bfloat16, dev, seed=7)
    lay = PagedKVLayout(kv)
    T, cs = 300, 128
    slots = block_slots(T, 16, 64, seed=8, device=dev)
    pin = dev == "cuda"
    chunks = []
    for n in (128, 128, 44):
        c = torch.zeros(lay.chunk_shape(n), dtype=torch.bfloat16)
        chunks.append(c.pin_memory() if pin else c)
    api.dense_mla_dsa_batched_direct_kv_transfer(chunks, lay, slots, cs, True)
    if pin:
        torch.cuda.synchronize()
    ref = torch.zeros(lay.chunk_shape(T), dtype=torch.bfloat16, device=dev)
    lay.gather_ref(ref, slots)
    assert torch.equal(torch.cat([c.to(dev) for c in chunks], dim=2), ref)


@pytest.mark.parametrize("dev", _devs())
def test_direct_fast_prepared_and_sparse_multi_chunk(dev):
    kv = make_separate_kv(2, 64, 16, 2, 64, torch.bfloat16, dev, seed=9)
    lay = PagedKVLayout(kv)
    T, cs = 256, 128
    slots = block_slots(T, 16, 64, seed=10, device=dev)
    pin = dev == "cuda"
    mk = lambda: [(lambda c: c.pin_memory() if pin else c)(
        torch.zeros(lay.chunk_shape(cs), dtype=torch.bfloat16)) for _ in range(T // cs)]
    ref = torch.zeros(lay.chunk_shape(T), dtype=torch.bfloat16, device=dev)
    lay.gather_ref(ref, slots)
    a, b = mk(), mk()
    api.dense_mla_dsa_batched_direct_kv_transfer_fast(a, lay, slots, cs, True)
    api.dense_mla_dsa_batched_direct_kv_transfer_fast(a, lay, slots, cs, True)  # cached state
    st = api.DirectTransferState(b, lay, cs)
    api.dense_mla_dsa_batched_direct_kv_transfer_prepared(st, slots, True)
    if pin:
        torch.cuda.synchronize()
    for got in (a, b):
        assert torch.equal(torch.cat([c.to(dev) for c in got], dim=2), ref)
    # sparse multi-chunk: scatter 50 selected tokens of the chunk sequence
    kv2 = [(torch.zeros_like(x), torch.zeros_like(y)) for x, y in kv]
    lay2 = PagedKVLayout(kv2)
    g = torch.Generator().manual_seed(11)
    sel = torch.randperm(T, generator=g)[:50]
    dst = random_slots(50, 64 * 16, seed=12, device=dev)
    api.mla_dsa_sparse_multi_chunk_kv_transfer(a, lay2, dst, sel.to(dev), cs)
    if pin:
        torch.cuda.synchronize()
    for layer in range(2):
        for plane in range(2):
            got = kv2[layer][plane].reshape(-1, 128)[dst.long()]
            assert torch.equal(got.cpu(), ref[plane, layer][sel].cpu())
    with pytest.raises(NotImplementedError):
        api.multi_layer_kv_transfer_unilateral()


@GPU
def test_sparse_graph_capture_replay():
    kv = make_separate_kv(1, 64, 16, 4, 64, torch.bfloat16, "cuda", seed=9)
    kv2 = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in kv]
    lay2 = PagedKVLayout(kv2)
    cap = 256
    staging = torch.randn(cap, 2, 256, device="cuda").to(torch.bfloat16)  # token-major
    sel = torch.zeros(cap, dtype=torch.int64, device="cuda")
    slots = torch.full((cap,), -1, dtype=torch.int64, device="cuda")
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    lay2.native()
    api._single_layer_layout(lay2, True)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        api.sparse_graph_kv_transfer(staging, lay2, 0, slots, sel, count)  # warm
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        api.sparse_graph_kv_transfer(staging, lay2, 0, slots, sel, count)
    for n in (17, 200):
        kv2[0][0].zero_()
        sel.copy_(torch.randperm(cap, device="cuda"))
        slots.copy_(random_slots(cap, 1024, seed=n, device="cuda"))
        count.fill_(n)
        g.replay()
        torch.cuda.synchronize()
        k2 = kv2[0][0].reshape(-1, 256)
        assert torch.equal(k2[slots[:n]], staging[sel[:n], 0])
        assert int(k2[slots[n:]].abs().sum()) == 0


@GPU
@pytest.mark.parametrize("quantized,factor,use_map", [(True, 1, False), (True, 2, False),
                                                      (True, 1, True), (False, 1, False)])
def test_indexer_c8_round_trip(quantized, factor, use_map):
    L, NB = 3, 16
    dev = "cuda"
    states = []
    for l in range(L):
        if quantized:
            keys = torch.randint(-128, 127, (NB, 128, 1, 128), dtype=torch.int8, device=dev)
            scales = torch.randn(NB, 128, 1, 1, device=dev).to(torch.float16)
        else:
            keys = torch.randn(NB, 128, 1, 128, device=dev).to(torch.bfloat16)
            scales = None
        bmap = torch.randperm(NB, device=dev).to(torch.int32) if use_map else None
        states.append(api.IndexerC8State(keys, scales, factor, bmap))
    group = api.IndexerC8GroupState(states)
    cap, T = 256, 300
    slots = random_slots(T, states[0].cache_slots, seed=10, device=dev)
    sizes = [256, 44]
    packets = [torch.zeros(group.packet_bytes(n), dtype=torch.uint8, device=dev) for n in sizes]
    api.indexer_c8_transfer_prepared(group, packets, slots, cap, from_gpu=True)
    torch.cuda.synchronize()
    s = 0
    for p, n in zip(packets, sizes):
        assert torch.equal(p.cpu(), api.indexer_c8_packets_ref(group, slots[s:s + n], n))
        s += n
    # back into zeroed caches
    states2 = [api.IndexerC8State(torch.zeros_like(st.keys),
                                  None if st.scales is None else torch.zeros_like(st.scales),
                                  factor, st.block_map) for st in states]
    g2 = api.IndexerC8GroupState(states2)
    api.indexer_c8_transfer_prepared(g2, packets, slots, cap, from_gpu=False)
    torch.cuda.synchronize()
    phys = states[0].physical_slots(slots)
    for a, b in zip(states, states2):
        ka = a.keys.view(-1, 128)[phys]
        kb = b.keys.view(-1, 128)[phys]
        assert torch.equal(ka, kb)
        if quantized:
            assert torch.equal(a.scales.view(-1)[phys], b.scales.view(-1)[phys])
