"""K9 PD push: byte-exact paged->paged push, per-layer flags, bounded wait.

Single-GPU tests run the push in loopback (sender and receiver caches on one
device; same kernel, local instead of peer addresses).  The timeout test
waits on a flag that nothing sets and checks the reported status: the wait is
bounded (0.2 s) and the context stays usable.
"""

import pytest
import torch

from lmcache_ascend_b200.parallel.pd_push import PushReceiver, PushSender
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

from .utils import block_slots, make_mla_kv, make_separate_kv, random_slots

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rows(kv, slots):
    s = slots.long()
    out = []
    for layer in kv:
        for t in layer:
            out.append(t.view(t.shape[0] * t.shape[1], -1)[s])
    return out


@pytest.mark.parametrize("pattern", ["blocks", "random"])
@pytest.mark.parametrize("tile", [32, 128])
@pytest.mark.parametrize("engine", ["auto", "bulk", "simt"])
def test_loopback_push_exact(pattern, tile, engine):
    L, NB, BS = 6, 32, 128
    src = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=1)
    dst = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=2)
    T = 1000
    if pattern == "blocks":
        ss = block_slots(T, BS, NB, seed=3, device=DEV, dtype=torch.int32)
        ds = block_slots(T, BS, NB, seed=4, device=DEV, dtype=torch.int32)
    else:
        ss = random_slots(T, NB * BS, seed=5, device=DEV, dtype=torch.int32)
        ds = random_slots(T, NB * BS, seed=6, device=DEV, dtype=torch.int32)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src), engine=engine)
    send.connect([recv.desc])
    tg = recv.expect(T, tile_tokens=tile)
    send.push(ss, ds, tile_tokens=tile)
    recv.wait(tg, timeout_s=2.0)
    torch.cuda.synchronize()
    send.check()
    recv.check()
    for a, b in zip(_rows(src, ss), _rows(dst, ds)):
        assert torch.equal(a, b)
    # flags: units per layer = planes * ceil(T / tile)
    per_layer = 2 * ((T + tile - 1) // tile)
    assert recv.flags[:L].tolist() == [per_layer] * L


def test_layerwise_push_and_partial_wait():
    L, NB, BS = 4, 16, 128
    src = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=7)
    dst = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=8)
    T = 512
    ss = block_slots(T, BS, NB, seed=9, device=DEV, dtype=torch.int32)
    ds = block_slots(T, BS, NB, seed=10, device=DEV, dtype=torch.int32)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src), engine="auto")
    send.connect([recv.desc])
    for layer in range(L):
        tg = recv.expect(T, layer_begin=layer, num_layers=1)
        send.push(ss, ds, layer_begin=layer, num_layers=1)
        recv.wait(tg, layer_begin=layer, timeout_s=2.0)
    torch.cuda.synchronize()
    recv.check()
    for a, b in zip(_rows(src, ss), _rows(dst, ds)):
        assert torch.equal(a, b)


def test_fanout_two_replicas_mla():
    L, NB, BS = 3, 16, 64
    src = make_mla_kv(L, NB, BS, 512, 64, torch.bfloat16, DEV, seed=11)
    d1 = make_mla_kv(L, NB, BS, 512, 64, torch.bfloat16, DEV, seed=12)
    d2 = make_mla_kv(L, NB, BS, 512, 64, torch.bfloat16, DEV, seed=13)
    T = 300
    ss = random_slots(T, NB * BS, seed=14, device=DEV, dtype=torch.int64)
    ds = random_slots(T, NB * BS, seed=15, device=DEV, dtype=torch.int64)
    r1 = PushReceiver(PagedKVLayout(d1, use_mla=True))
    r2 = PushReceiver(PagedKVLayout(d2, use_mla=True))
    send = PushSender(PagedKVLayout(src, use_mla=True))
    send.connect([r1.desc, r2.desc])
    t1, t2 = r1.expect(T), r2.expect(T)
    send.push(ss, ds)
    r1.wait(t1, timeout_s=2.0)
    r2.wait(t2, timeout_s=2.0)
    torch.cuda.synchronize()
    r1.check()
    r2.check()
    for a, b, c in zip(_rows(src, ss), _rows(d1, ds), _rows(d2, ds)):
        assert torch.equal(a, b) and torch.equal(a, c)


def test_wait_times_out_with_status():
    dst = make_separate_kv(2, 4, 16, 1, 64, torch.bfloat16, DEV)
    recv = PushReceiver(PagedKVLayout(dst))
    tg = recv.expect(64)  # nothing will ever push
    recv.wait(tg, timeout_s=0.2)
    torch.cuda.synchronize()
    st = recv.status.read()
    assert st["name"] == "flag_timeout"
    # the context is still usable
    x = torch.ones(4, device=DEV) * 2
    assert float(x.sum()) == 8.0


def _fp8_ref(rows: torch.Tensor, group: int) -> torch.Tensor:
    """PyTorch reference of the block-scaled fp8 round trip of bf16 rows."""
    x = rows.float().view(rows.shape[0], -1, group)
    amax = x.abs().amax(dim=-1, keepdim=True)
    # IEEE fp32 quotients (PyTorch divides by a scalar through its reciprocal):
    # a float64 quotient rounded once to fp32 is the correctly rounded one
    inv = torch.where(amax > 0, (448.0 / amax.double()).float(), torch.zeros_like(amax))
    # a group too small for a finite inverse scale is sent as zeros, scale 0
    tiny = torch.isinf(inv)
    inv = torch.where(tiny, torch.zeros_like(inv), inv)
    scale = torch.where(tiny, torch.zeros_like(amax), (amax.double() / 448.0).float())
    q = (x * inv).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return (q.float() * scale).to(torch.bfloat16).view_as(rows)


@pytest.mark.parametrize("group", [128, 256])
@pytest.mark.parametrize("tile", [64, 128])
def test_fp8_push_matches_reference_and_halves_bytes(group, tile):
    L, NB, BS, H, D = 4, 32, 128, 2, 128
    src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=11)
    dst = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=12)
    src[1][0][3] = 0  # an all-zero block: scale 0
    # a block of bf16 subnormals (amax below 448 / FLT_MAX): zeros, not NaN
    src[2][1][5] = torch.full_like(src[2][1][5], 1e-38)
    src[2][1][5][::3] = 0
    T = 900
    ss = block_slots(T, BS, NB, seed=13, device=DEV, dtype=torch.int32)
    ds = random_slots(T, NB * BS, seed=14, device=DEV, dtype=torch.int32)
    recv = PushReceiver(PagedKVLayout(dst), fp8_staging_tokens=1024, fp8_group=group)
    send = PushSender(PagedKVLayout(src), engine="auto")
    send.connect([recv.desc])
    tg = recv.expect(T, tile_tokens=tile)
    send.push(ss, ds, tile_tokens=tile, quant="fp8")
    recv.wait(tg, timeout_s=2.0)
    recv.dequantize(ds)
    torch.cuda.synchronize()
    send.check()
    recv.check()
    for a, b in zip(_rows(src, ss), _rows(dst, ds)):
        assert not bool(torch.isnan(b).any())
        assert torch.equal(b, _fp8_ref(a, group))
        # bounded error: at most 2^-4 of the group's amax per element
        err = (b.float() - a.float()).view(T, -1, group).abs()
        bound = a.float().view(T, -1, group).abs().amax(-1, keepdim=True) * (2 ** -4) + 1e-2
        assert bool((err <= bound).all())
    wire = recv._fp8_qb + recv._fp8_sb  # one staging buffer = one request's bytes
    assert wire < 0.56 * 1024 * L * 2 * H * D * 2  # about half the bf16 bytes


def test_fp8_requests_rotate_through_staging_buffers():
    """Five fp8 requests in a row through two staging buffers: each is
    dequantised from the buffer it was written to, and every wait on a
    released buffer completes (no timeout reported)."""
    L, NB, BS, H, D = 2, 16, 128, 2, 128
    dst = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=21)
    recv = PushReceiver(PagedKVLayout(dst), fp8_staging_tokens=512, fp8_buffers=2)
    T = 300
    src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=30)
    send = PushSender(PagedKVLayout(src), engine="auto")
    send.connect([recv.desc])
    for i in range(5):
        g = torch.Generator(device=DEV).manual_seed(70 + i)
        for layer in src:
            for plane in layer:
                plane.copy_(torch.randn(plane.shape, generator=g, device=DEV))
        ss = block_slots(T, BS, NB, seed=40 + i, device=DEV, dtype=torch.int32)
        ds = random_slots(T, NB * BS, seed=50 + i, device=DEV, dtype=torch.int32)
        tg = recv.expect(T)
        send.push(ss, ds, quant="fp8", staging_timeout_s=2.0)
        for l0 in range(L):  # one layer at a time; the last one releases
            recv.wait(tg[l0:l0 + 1], layer_begin=l0, timeout_s=2.0)
            recv.dequantize(ds, layer_begin=l0, num_layers=1)
        torch.cuda.synchronize()
        send.check()
        recv.check()
        for a, b in zip(_rows(src, ss), _rows(dst, ds)):
            assert torch.equal(b, _fp8_ref(a, 128))
    send.close()
    assert recv._fp8_seq == 5 and send._fp8_seq == 5


def test_fp8_staging_not_released_reports_timeout():
    """The receiver never dequantises: the sender's third request finds no
    free staging buffer and its bounded wait reports a flag timeout."""
    L, NB, BS, H, D = 2, 16, 128, 2, 128
    src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=61)
    dst = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, DEV, seed=62)
    recv = PushReceiver(PagedKVLayout(dst), fp8_staging_tokens=256, fp8_buffers=2)
    send = PushSender(PagedKVLayout(src), engine="auto")
    send.connect([recv.desc])
    ss = block_slots(200, BS, NB, seed=63, device=DEV, dtype=torch.int32)
    send.push(ss, ss, quant="fp8", staging_timeout_s=0.2)
    send.push(ss, ss, quant="fp8", staging_timeout_s=0.2)
    torch.cuda.synchronize()
    send.check()  # two buffers: no wait yet
    send.push(ss, ss, quant="fp8", staging_timeout_s=0.2)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError):
        send.check()
    send.close()


def test_fp8_push_rejects_planes_of_4gib():
    """The fp8 push addresses rows with 32-bit offsets inside a layer plane:
    a layout whose plane spans 4 GiB or more is refused before any launch
    (the layout below only describes such a plane; nothing is allocated)."""
    from lmcache_ascend_b200 import ops

    nb, bs, rb = 1 << 16, 128, 512            # 65536 blocks x 64 KiB = 4 GiB
    ptrs = torch.full((2,), 1 << 40, dtype=torch.int64, device=DEV)
    lay = ops.native().PagedLayout(ptrs, [bs * rb, bs * rb], [rb, rb], [rb, rb], bs, nb * bs,
                                   [], [])
    slots = torch.zeros(16, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="4 GiB"):
        ops.native().pd_push_fp8(lay, 0, 0, slots, 0, 1, 0, 128, 0, 128, None)


@pytest.mark.parametrize("grid", [1, 3, 7])
@pytest.mark.parametrize("tile", [32, 512])
def test_bulk_push_units_shared_between_warps(grid, tile):
    """Small grids give every warp a long range of pieces, so units are split
    between warps and published by whichever finishes last (per-unit
    counters); three pushes in a row check the counters return to zero."""
    L, NB, BS = 3, 32, 128
    src = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=31)
    dst = make_separate_kv(L, NB, BS, 2, 128, torch.bfloat16, DEV, seed=32)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src), engine="bulk")
    send.connect([recv.desc])
    T = 1777
    for i in range(3):
        for layer in src:
            for t in layer:
                t.normal_()
        ss = random_slots(T, NB * BS, seed=40 + i, device=DEV, dtype=torch.int32)
        ds = block_slots(T, BS, NB, seed=50 + i, device=DEV, dtype=torch.int32)
        tg = recv.expect(T, tile_tokens=tile)
        send.push(ss, ds, tile_tokens=tile, grid=grid)
        recv.wait(tg, timeout_s=2.0)
        torch.cuda.synchronize()
        send.check()
        recv.check()
        for a, b in zip(_rows(src, ss), _rows(dst, ds)):
            assert torch.equal(a, b)
    per_layer = 2 * ((T + tile - 1) // tile)
    assert recv.flags[:L].tolist() == [3 * per_layer] * L
    assert int(send._counters.abs().sum()) == 0
    send.close()


def test_bulk_push_c8_planes_fused():
    """A DSA-style layer of three planes with different row sizes (1152-byte
    latent, 128-byte int8 indexer key, 4-byte fp32 scale) in ONE bulk push
    launch: the 4-byte plane rides per lane inside the same kernel."""
    L, NB, BS = 3, 32, 64

    def cache(seed):
        g = torch.Generator(device=DEV).manual_seed(seed)
        out = []
        for _ in range(L):
            lat = torch.randn(NB, BS, 576, generator=g, device=DEV).to(torch.bfloat16)
            key = torch.randint(-128, 128, (NB, BS, 128), generator=g, device=DEV,
                                dtype=torch.int8)
            sc = torch.rand(NB, BS, 1, generator=g, device=DEV)
            out.append(tuple(t.view(torch.uint8).view(NB, BS, -1) for t in (lat, key, sc)))
        return out

    src, dst = cache(1), cache(2)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src))
    send.connect([recv.desc])
    T = 1000
    ss = random_slots(T, NB * BS, seed=3, device=DEV, dtype=torch.int32)
    ds = random_slots(T, NB * BS, seed=4, device=DEV, dtype=torch.int32)
    tg = recv.expect(T)
    send.push(ss, ds)
    recv.wait(tg, timeout_s=2.0)
    torch.cuda.synchronize()
    send.check()
    recv.check()
    for ls, ld in zip(src, dst):
        for a, b in zip(ls, ld):
            assert torch.equal(a.reshape(NB * BS, -1)[ss.long()],
                               b.reshape(NB * BS, -1)[ds.long()])
