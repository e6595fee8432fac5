"""The reference-signature op table (``lmcache_ascend_b200.c_ops``) against
direct PyTorch indexing of the caches (exact copies): pointer tables built the way the
reference connector builds them, chunks checked byte for byte."""

import pytest
import torch

from .utils import block_slots, make_separate_kv

pytestmark = pytest.mark.gpu

L, NB, BS, H, D = 3, 16, 16, 2, 64
T = 200


def _rows(t, slots):
    return t.reshape(NB * BS, -1)[slots.long()]


@pytest.mark.parametrize("direction", [True, False])
def test_multi_layer_separate_table(direction):
    from lmcache_ascend_b200 import c_ops

    kv = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=1)
    ptrs = torch.tensor([t.data_ptr() for k, v in kv for t in (k, v)], dtype=torch.int64,
                        device="cuda")
    slots = block_slots(T, BS, NB, seed=2, device="cuda")
    chunk = torch.randn(2, L, T, H * D, device="cuda").to(torch.bfloat16)
    c_ops.multi_layer_kv_transfer(chunk, ptrs, slots, torch.device("cuda"), NB * BS, direction,
                                  False, c_ops.SEPARATE_KV)
    torch.cuda.synchronize()
    for l, (k, v) in enumerate(kv):
        assert torch.equal(chunk[0, l], _rows(k, slots))
        assert torch.equal(chunk[1, l], _rows(v, slots))


def test_multi_layer_merged_two_major_host_chunk():
    from lmcache_ascend_b200 import c_ops

    caches = [torch.randn(2, NB, BS, H, D, device="cuda").to(torch.bfloat16) for _ in range(L)]
    ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64, device="cuda")
    slots = block_slots(T, BS, NB, seed=3, device="cuda")
    chunk = torch.zeros(2, L, T, H * D, dtype=torch.bfloat16).pin_memory()
    c_ops.multi_layer_kv_transfer(chunk, ptrs, slots, "cuda", NB * BS, True)
    torch.cuda.synchronize()
    for l, c in enumerate(caches):
        assert torch.equal(chunk[0, l].cuda(), _rows(c[0], slots))
        assert torch.equal(chunk[1, l].cuda(), _rows(c[1], slots))


def test_multi_layer_mla_two_planes():
    from lmcache_ascend_b200 import c_ops

    lat, rope = 128, 32
    planes = [(torch.randn(NB, BS, lat, device="cuda").to(torch.bfloat16),
               torch.randn(NB, BS, rope, device="cuda").to(torch.bfloat16)) for _ in range(L)]
    ptrs = torch.tensor([t.data_ptr() for p in planes for t in p], dtype=torch.int64,
                        device="cuda")
    slots = block_slots(T, BS, NB, seed=4, device="cuda")
    chunk = torch.zeros(1, L, T, lat + rope, dtype=torch.bfloat16, device="cuda")
    c_ops.multi_layer_kv_transfer(chunk, ptrs, slots, "cuda", NB * BS, True, True,
                                  c_ops.MLA_KV, lat, rope, 0)
    torch.cuda.synchronize()
    for l, (a, b) in enumerate(planes):
        assert torch.equal(chunk[0, l, :, :lat], _rows(a, slots))
        assert torch.equal(chunk[0, l, :, lat:], _rows(b, slots))


def test_single_layer_and_flash_round_trip():
    from lmcache_ascend_b200 import c_ops

    kv = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=5)
    slots = block_slots(T, BS, NB, seed=6, device="cuda")
    buf = torch.randn(2, T, H * D, device="cuda").to(torch.bfloat16)
    k, v = kv[1]
    c_ops.single_layer_kv_transfer(buf, [k, v], slots, False, c_ops.SEPARATE_KV)
    torch.cuda.synchronize()
    assert torch.equal(_rows(k, slots), buf[0]) and torch.equal(_rows(v, slots), buf[1])

    chunk = torch.zeros(2, L, T, H * D, dtype=torch.bfloat16, device="cuda")
    for l, (k, v) in enumerate(kv):
        c_ops.reshape_and_cache_back_flash(chunk, k, v, slots, l)
    torch.cuda.synchronize()
    for l, (k, v) in enumerate(kv):
        assert torch.equal(chunk[0, l], _rows(k, slots))
        assert torch.equal(chunk[1, l], _rows(v, slots))
    fresh = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in kv]
    for l, (k, v) in enumerate(fresh):
        c_ops.load_and_reshape_flash(chunk, k, v, slots, l)
    torch.cuda.synchronize()
    for (k, v), (k2, v2) in zip(kv, fresh):
        assert torch.equal(_rows(k, slots), _rows(k2, slots))
        assert torch.equal(_rows(v, slots), _rows(v2, slots))
