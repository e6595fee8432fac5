"""K8 fused RoPE re-rotation vs an fp32 PyTorch reference (reference test
shapes: tests/v1/test_pos_kernels.py:319-342 -- D in {64, 128}, theta 500000,
neox both, bf16/fp32, T in {512, 1024, 4096})."""

import pytest
import torch

from lmcache_ascend_b200 import ops
from lmcache_ascend_b200.ops import reference as R


def test_reference_delta_equals_reapply():
    # rotating rope(old) by (new - old) == rope(new) of the raw key (fp32/fp64)
    T, H, D = 64, 4, 64
    cache = R.make_cos_sin_cache(4096, D, base=10000.0, dtype=torch.float64)
    k = torch.randn(T, H * D, dtype=torch.float64)
    old = torch.randint(0, 4000, (T,))
    new = torch.randint(0, 4000, (T,))
    for neox in (True, False):
        at_old = R.rope_apply_ref(old, k, D, cache, neox).double()
        moved = R.rope_delta_ref(old, new, at_old, D, cache, neox).double()
        direct = R.rope_apply_ref(new, k, D, cache, neox).double()
        assert torch.allclose(moved, direct, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("head_size", [64, 128])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T", [512, 1024, 4096])
def test_fused_rope_gpu(head_size, neox, dtype, T):
    H = 8
    cache = R.make_cos_sin_cache(8192 + T, head_size, base=500000.0).cuda()
    k = torch.randn(T, H * head_size, device="cuda").to(dtype)
    old = torch.randint(0, 8192, (T,), device="cuda")
    new = old + torch.randint(0, T, (T,), device="cuda")
    ref = R.rope_delta_ref(old.cpu(), new.cpu(), k.cpu(), head_size, cache.cpu(), neox)
    kk = k.clone()
    ops.native().rotary_embedding_k_fused(old, new, kk, head_size, cache, neox)
    torch.cuda.synchronize()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert torch.allclose(kk.float().cpu(), ref, atol=tol * 4, rtol=tol)


@pytest.mark.gpu
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rot", [128, 64])
def test_fused_rope_vector_path_matches_scalar_path(neox, dtype, rot):
    # the same keys once 16-byte aligned (vector kernel) and once shifted by
    # one element (scalar kernel): results must be identical
    T, H, D = 1000, 4, 128
    cache = R.make_cos_sin_cache(4096, rot, base=10000.0).cuda()
    k = torch.randn(T, H * D, device="cuda").to(dtype)
    old = torch.randint(0, 2048, (T,), device="cuda")
    new = old + torch.randint(0, 2048, (T,), device="cuda")
    a = k.clone()
    big = torch.zeros(T, H * D + 1, device="cuda", dtype=dtype)
    big[:, 1:] = k
    b = big[:, 1:]
    ops.native().rotary_embedding_k_fused(old, new, a, D, cache, neox)
    ops.native().rotary_embedding_k_fused(old, new, b, D, cache, neox)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    ref = R.rope_delta_ref(old.cpu(), new.cpu(), k.cpu(), D, cache.cpu(), neox)
    tol = 1e-2 if dtype != torch.float32 else 1e-5
    assert torch.allclose(a.float().cpu(), ref, atol=tol * 4, rtol=tol)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_rope_on_paged_mla_rope_part_by_slot(dtype):
    """CacheBlend on a paged MLA latent cache: only the 64 rope dims of each
    576-element row rotate, rows addressed by slot (slot -1 skipped), the
    512 latent dims and untouched slots stay bit-identical."""
    NB, BS, T = 64, 64, 700
    lat = torch.randn(NB, BS, 576, device="cuda").to(dtype)
    before = lat.clone()
    flat = lat.view(NB * BS, 576)
    key = flat[:, 512:]  # [rows, 64], row stride 576
    slots = torch.randperm(NB * BS, device="cuda")[:T]
    slots[::9] = -1
    cache = R.make_cos_sin_cache(16384, 64, base=10000.0).cuda()
    old = torch.randint(0, 8192, (T,), device="cuda")
    new = old + torch.randint(0, 8192, (T,), device="cuda")
    ops.native().rotary_embedding_k_fused(old, new, key, 64, cache, True, slots)
    torch.cuda.synchronize()
    keep = slots >= 0
    s = slots[keep]
    ref = R.rope_delta_ref(old[keep].cpu(), new[keep].cpu(),
                           before.view(NB * BS, 576)[s, 512:].cpu(), 64, cache.cpu(), True)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    got = lat.view(NB * BS, 576)
    assert torch.allclose(got[s, 512:].float().cpu(), ref, atol=tol * 4, rtol=tol)
    assert torch.equal(got[:, :512], before.view(NB * BS, 576)[:, :512])
    untouched = torch.ones(NB * BS, dtype=torch.bool, device="cuda")
    untouched[s] = False
    assert torch.equal(got[untouched], before.view(NB * BS, 576)[untouched])
    # the CPU oracle path of the op gives the same rows
    cpu = before.view(NB * BS, 576).cpu().clone()
    from lmcache_ascend_b200.ops import api

    api.rotary_embedding_k_fused(old.cpu(), new.cpu(), cpu[:, 512:], 64, cache.cpu(), True,
                                 slots.cpu())
    assert torch.allclose(got.float().cpu(), cpu.float(), atol=tol * 4, rtol=tol)


@pytest.mark.gpu
def test_fused_rope_several_layers_in_one_launch_matches_per_layer():
    """The multi-layer form (every layer's rope columns of a paged MLA cache
    in one launch) leaves the same bits as one call per layer, and matches
    the fp32 PyTorch oracle."""
    L, NB, BS, T = 5, 32, 64, 900
    g = torch.Generator(device="cpu").manual_seed(3)
    lats = [torch.randn(NB, BS, 576, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    twins = [x.clone() for x in lats]
    before = [x.clone() for x in lats]
    slots = torch.randperm(NB * BS, generator=g)[:T].int().cuda()
    slots[::7] = -1
    cache = R.make_cos_sin_cache(16384, 64, base=10000.0).cuda()
    old = torch.randint(0, 8192, (T,), generator=g).int().cuda()
    new = old + torch.randint(0, 8192, (T,), generator=g).int().cuda()
    keys = [x.view(NB * BS, 576)[:, 512:] for x in lats]
    ops.native().rotary_embedding_k_fused_layers(old, new, keys, 64, cache, True, slots)
    for x in twins:
        ops.native().rotary_embedding_k_fused(old, new, x.view(NB * BS, 576)[:, 512:], 64,
                                              cache, True, slots)
    torch.cuda.synchronize()
    keep = slots >= 0
    s = slots[keep].long()
    for x, y, b in zip(lats, twins, before):
        assert torch.equal(x, y)
        ref = R.rope_delta_ref(old[keep].long().cpu(), new[keep].long().cpu(),
                               b.view(NB * BS, 576)[s, 512:].cpu(), 64, cache.cpu(), True)
        got = x.view(NB * BS, 576)[s, 512:].float().cpu()
        assert torch.allclose(got, ref, atol=4e-2, rtol=1e-2)
