"""K1/K2/K3/K4/K5 gather/scatter kernels vs the PyTorch oracle (bit-exact).

Covers every paged format, both engines (TMA bulk and SIMT), single and
multi-chunk (pointer table) views, device and host-mapped pinned chunks,
sparse chunk indices, device-side token counts and bad-slot reporting.
"""

import pytest
import torch

from lmcache_ascend_b200 import ops
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

from .utils import block_slots, make_merged_kv, make_mla_kv, make_separate_kv, random_slots

pytestmark = pytest.mark.gpu

DEV = "cuda"
TMA, SIMT = 1, 2


def _kv(fmt, dtype=torch.bfloat16, L=4, NB=64, BS=16):
    if fmt == "separate":
        return make_separate_kv(L, NB, BS, 8, 128, dtype, DEV), False
    if fmt == "merged":
        return make_merged_kv(L, NB, BS, 4, 64, dtype, DEV), False
    if fmt == "flashinfer":
        return make_merged_kv(L, NB, BS, 4, 64, dtype, DEV, flashinfer=True), False
    if fmt == "mla":
        return make_mla_kv(L, NB, BS, 512, 64, dtype, DEV), True
    if fmt == "mla_flat":
        return make_mla_kv(L, NB, BS, 512, 64, dtype, DEV, flat=True), True
    if fmt == "dsa":
        return make_mla_kv(L, NB, BS, 512, 64, dtype, DEV, indexer_dim=128), True
    raise ValueError(fmt)


def _xfer(layout, chunk, slots, to_chunk, mode, **kw):
    ops.native().kv_transfer(layout.native(), chunk, kw.pop("chunk_ptrs", None),
                             layout.chunk_native(), kw.pop("ntok", chunk.shape[2]
                                                           if chunk is not None else 0),
                             kw.pop("tok_off", 0), kw.pop("chunk_tokens", 0),
                             kw.pop("on_device", True), slots, 0, 0, layout.num_layers,
                             to_chunk, mode, kw.pop("status", None), kw.pop("chunk_idx", None),
                             kw.pop("chunk_idx_limit", 0), kw.pop("num_tokens_dev", None))


@pytest.mark.parametrize("fmt", ["separate", "merged", "flashinfer", "mla", "mla_flat", "dsa"])
@pytest.mark.parametrize("mode", [TMA, SIMT])
@pytest.mark.parametrize("pattern", ["blocks", "random", "holes"])
def test_gather_scatter_exact(fmt, mode, pattern):
    kv, mla = _kv(fmt)
    lay = PagedKVLayout(kv, use_mla=mla)
    T = 300
    if pattern == "blocks":
        slots = block_slots(T, lay.block_size, lay.num_blocks, seed=1, device=DEV)
    else:
        slots = random_slots(T, lay.num_slots, seed=2, device=DEV)
    if pattern == "holes":
        slots[::7] = -1
    # gather
    got = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype, device=DEV)
    ref = torch.zeros_like(got)
    _xfer(lay, got, slots, True, mode)
    lay.gather_ref(ref, slots)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    # scatter into a fresh cache
    src = torch.randn(lay.chunk_shape(T), device=DEV).to(lay.dtype)
    kv2 = [tuple(torch.zeros_like(t) for t in l) if isinstance(l, tuple) else torch.zeros_like(l)
           for l in kv]
    kv3 = [tuple(torch.zeros_like(t) for t in l) if isinstance(l, tuple) else torch.zeros_like(l)
           for l in kv]
    lay2, lay3 = PagedKVLayout(kv2, use_mla=mla), PagedKVLayout(kv3, use_mla=mla)
    _xfer(lay2, src, slots, False, mode)
    lay3.scatter_ref(src, slots)
    torch.cuda.synchronize()
    for a, b in zip(kv2, kv3):
        if isinstance(a, tuple):
            for x, y in zip(a, b):
                assert torch.equal(x, y)
        else:
            assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_dtypes(dtype):
    kv, _ = _kv("separate", dtype=dtype)
    lay = PagedKVLayout(kv)
    slots = block_slots(256, 16, 64, seed=3, device=DEV)
    got = torch.zeros(lay.chunk_shape(256), dtype=dtype, device=DEV)
    ref = torch.zeros_like(got)
    _xfer(lay, got, slots, True, 0)
    lay.gather_ref(ref, slots)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("on_device", [True, False])
def test_multi_chunk_table(on_device):
    kv, _ = _kv("separate")
    lay = PagedKVLayout(kv)
    cs, T = 128, 300  # 3 chunks, last partial
    slots = block_slots(T, 16, 64, seed=4, device=DEV)
    sizes = [128, 128, 44]
    if on_device:
        chunks = [torch.zeros(lay.chunk_shape(n), dtype=lay.dtype, device=DEV) for n in sizes]
    else:
        chunks = [torch.zeros(lay.chunk_shape(n), dtype=lay.dtype).pin_memory() for n in sizes]
    ptrs = torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64, device=DEV)
    _xfer(lay, None, slots, True, TMA if on_device else SIMT, chunk_ptrs=ptrs, chunk_tokens=cs,
          on_device=on_device)
    torch.cuda.synchronize()
    s = 0
    for c, n in zip(chunks, sizes):
        ref = torch.zeros(lay.chunk_shape(n), dtype=lay.dtype, device=DEV)
        lay.gather_ref(ref, slots[s:s + n])
        assert torch.equal(c.to(DEV), ref)
        s += n
    # and back (scatter) into a zeroed cache
    kv2 = [tuple(torch.zeros_like(t) for t in l) for l in kv]
    lay2 = PagedKVLayout(kv2)
    _xfer(lay2, None, slots, False, TMA if on_device else SIMT, chunk_ptrs=ptrs,
          chunk_tokens=cs, on_device=on_device)
    torch.cuda.synchronize()
    idx = slots.long()
    for (k, v), (k2, v2) in zip(kv, kv2):
        assert torch.equal(k.view(-1, 1024)[idx], k2.view(-1, 1024)[idx])
        assert torch.equal(v.view(-1, 1024)[idx], v2.view(-1, 1024)[idx])


def test_sparse_chunk_index_and_device_count():
    kv, _ = _kv("separate")
    lay = PagedKVLayout(kv)
    T = 256
    src = torch.randn(lay.chunk_shape(T), device=DEV).to(lay.dtype)
    n_sel = 100
    sel = torch.randperm(T, device=DEV)[:n_sel].to(torch.int64)
    slots = random_slots(n_sel, lay.num_slots, seed=5, device=DEV)
    count = torch.tensor([60], dtype=torch.int32, device=DEV)  # only the first 60
    kv2 = [tuple(torch.zeros_like(t) for t in l) for l in kv]
    lay2 = PagedKVLayout(kv2)
    _xfer(lay2, src, slots, False, TMA, chunk_idx=sel, chunk_idx_limit=T,
          num_tokens_dev=count)
    torch.cuda.synchronize()
    for l, (k2, v2) in enumerate(kv2):
        kf = k2.view(-1, 1024)
        assert torch.equal(kf[slots[:60].long()], src[0, l][sel[:60]])
        assert int(kf[slots[60:].long()].abs().sum()) == 0


def test_bad_slot_reported_and_skipped():
    kv, _ = _kv("separate")
    lay = PagedKVLayout(kv)
    slots = block_slots(64, 16, 64, seed=6, device=DEV)
    slots[5] = lay.num_slots + 10  # out of range: must be skipped and reported
    st = ops.DeviceStatus(torch.device(DEV))
    got = torch.zeros(lay.chunk_shape(64), dtype=lay.dtype, device=DEV)
    _xfer(lay, got, slots, True, TMA, status=st.tensor)
    torch.cuda.synchronize()
    r = st.read()
    assert r["name"] == "bad_slot" and r["a"] == lay.num_slots + 10


@pytest.mark.parametrize("fmt", ["separate", "mla"])
def test_fused_staged_host_transfer(fmt):
    """from_gpu: gather -> staging -> D2H; to_gpu: H2D -> staging -> scatter."""
    kv, mla = _kv(fmt)
    lay = PagedKVLayout(kv, use_mla=mla)
    T = 256
    slots = block_slots(T, lay.block_size, lay.num_blocks, seed=8, device=DEV)
    host = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype).pin_memory()
    staging = torch.empty(lay.chunk_bytes(T) + 4096, dtype=torch.uint8, device=DEV)
    ops.native().fused_multi_layer_kv_transfer(host, staging, lay.native(), lay.chunk_native(),
                                               slots, True)
    torch.cuda.synchronize()
    ref = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype, device=DEV)
    lay.gather_ref(ref, slots)
    assert torch.equal(host, ref.cpu())
    kv2 = [tuple(torch.zeros_like(t) for t in l) if isinstance(l, tuple) else torch.zeros_like(l)
           for l in kv]
    lay2 = PagedKVLayout(kv2, use_mla=mla)
    ops.native().fused_multi_layer_kv_transfer(host, staging, lay2.native(), lay2.chunk_native(),
                                               slots, False)
    torch.cuda.synchronize()
    back = torch.zeros_like(ref)
    lay2.gather_ref(back, slots)
    assert torch.equal(back, ref)


def _hnd_cache(L, NB, BS, H, D, seed):
    """flashinfer-style [NB, 2, BS, H, D] view over head-major [NB, 2, H, BS, D] storage"""
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(NB, 2, H, BS, D, generator=g).to(torch.bfloat16).to(DEV)
            .permute(0, 1, 3, 2, 4) for _ in range(L)]


@pytest.mark.parametrize("mode", [0, SIMT])
def test_head_major_layout_gather_scatter(mode):
    kv = _hnd_cache(3, 32, 16, 4, 64, seed=11)
    lay = PagedKVLayout(kv)
    assert lay.planes[0].segmented and lay.native().segmented
    T = 200
    slots = random_slots(T, lay.num_slots, seed=12, device=DEV)
    got = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype, device=DEV)
    ref = torch.zeros_like(got)
    _xfer(lay, got, slots, True, mode)
    lay.gather_ref(ref, slots)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    kv2 = [torch.zeros_like(t) for t in kv]
    lay2 = PagedKVLayout(kv2)
    _xfer(lay2, got, slots, False, mode)
    torch.cuda.synchronize()
    back = torch.zeros_like(ref)
    lay2.gather_ref(back, slots)
    assert torch.equal(back, ref)


@pytest.mark.parametrize("engine", ["auto", "simt"])
def test_head_major_push(engine):
    from lmcache_ascend_b200.parallel.pd_push import PushReceiver, PushSender

    src = _hnd_cache(2, 16, 16, 4, 64, seed=13)
    dst = [torch.zeros_like(t) for t in src]
    T = 150
    ss = random_slots(T, 256, seed=14, device=DEV, dtype=torch.int32)
    ds = random_slots(T, 256, seed=15, device=DEV, dtype=torch.int32)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src), engine=engine)
    send.connect([recv.desc])
    tg = recv.expect(T)
    send.push(ss, ds)
    recv.wait(tg, timeout_s=2.0)
    torch.cuda.synchronize()
    send.check()
    recv.check()
    ls, ld = PagedKVLayout(src), PagedKVLayout(dst)
    a = torch.zeros(ls.chunk_shape(T), dtype=ls.dtype, device=DEV)
    b = torch.zeros_like(a)
    ls.gather_ref(a, ss)
    ld.gather_ref(b, ds)
    assert torch.equal(a, b)
