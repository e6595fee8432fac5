"""The allocation-free C entry point `lmc_staged_kv_transfer_noalloc`.

Some callers cannot allocate device memory when they move KV: a serving
runtime that gave all free HBM to its KV cache, or a C host program with no
torch allocator and no tensor to offer as staging.  This entry point keeps
its staging buffer in a fixed device array inside the library, so the caller
passes only inputs and outputs.  The test calls it through its exported C
symbol (ctypes) and checks, on two calls in a row and in both directions,
that it produces exactly what the existing staged op
(`fused_multi_layer_kv_transfer`, caller-provided staging tensor) produces,
and exactly what the PyTorch oracle of the layout (`gather_ref` /
`scatter_ref`, plain indexing) produces.
It also checks that an oversized transfer is rejected with an error.
This file is named to be collected last.
"""

import ctypes

import pytest
import torch

from lmcache_ascend_b200 import ops
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

from .utils import block_slots, make_mla_kv, make_separate_kv

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    ops.native()  # loads the extension (and torch's CUDA libraries) first
    lib = ctypes.CDLL(ops.native_so_path())
    f = lib.lmc_staged_kv_transfer_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                  ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_char_p, ctypes.c_size_t]
    lib.lmc_noalloc_staging_capacity.restype = ctypes.c_size_t
    return lib


def _call(lib, lay: PagedKVLayout, slots: torch.Tensor, host: torch.Tensor, from_gpu: bool):
    n = lay.num_planes
    es = lay.elem_size
    ptrs = lay.native().ptrs  # device table of plane bases (caller's input)
    bs = (ctypes.c_int64 * n)(*[p.views[0].stride(0) * es for p in lay.planes])
    ss = (ctypes.c_int64 * n)(*[p.views[0].stride(1) * es for p in lay.planes])
    rb = (ctypes.c_int32 * n)(*lay.row_bytes)
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.lmc_staged_kv_transfer_noalloc(
        ptrs.data_ptr(), lay.num_layers, n, bs, ss, rb, lay.block_size, lay.num_slots,
        slots.data_ptr(), int(slots.dtype == torch.int64), slots.numel(), host.data_ptr(),
        host.numel() * host.element_size(), int(from_gpu), torch.cuda.current_device(),
        stream, err, len(err))
    return rc, err.value.decode()


def _fresh(kv):
    return [tuple(torch.zeros_like(t) for t in l) if isinstance(l, tuple) else torch.zeros_like(l)
            for l in kv]


@pytest.mark.parametrize("fmt", ["separate", "mla"])
def test_noalloc_matches_staged_op_two_calls(fmt):
    lib = _lib()
    if fmt == "separate":
        kv, mla = make_separate_kv(4, 64, 16, 8, 128, torch.bfloat16, DEV, seed=21), False
    else:
        kv, mla = make_mla_kv(4, 64, 16, 512, 64, torch.bfloat16, DEV, seed=22), True
    lay = PagedKVLayout(kv, use_mla=mla)
    for call, (T, seed) in enumerate([(256, 31), (200, 32)]):
        slots = block_slots(T, lay.block_size, lay.num_blocks, seed=seed, device=DEV,
                            dtype=torch.int32 if call else torch.int64)
        # store direction
        want = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype).pin_memory()
        staging = torch.empty(lay.chunk_bytes(T), dtype=torch.uint8, device=DEV)
        ops.native().fused_multi_layer_kv_transfer(want, staging, lay.native(),
                                                   lay.chunk_native(), slots, True)
        got = torch.full(lay.chunk_shape(T), 7, dtype=lay.dtype).pin_memory()
        rc, msg = _call(lib, lay, slots, got, True)
        torch.cuda.synchronize()
        assert rc == 0, msg
        assert torch.equal(got, want), f"store call {call}"
        oracle = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype)
        lay.gather_ref(oracle, slots)
        assert torch.equal(got, oracle), f"store call {call} vs the PyTorch oracle"
        # load direction, into two fresh caches
        kv_a, kv_b = _fresh(kv), _fresh(kv)
        lay_a, lay_b = PagedKVLayout(kv_a, use_mla=mla), PagedKVLayout(kv_b, use_mla=mla)
        ops.native().fused_multi_layer_kv_transfer(want, staging, lay_a.native(),
                                                   lay_a.chunk_native(), slots, False)
        rc, msg = _call(lib, lay_b, slots, want, False)
        torch.cuda.synchronize()
        assert rc == 0, msg
        kv_c = _fresh(kv)
        PagedKVLayout(kv_c, use_mla=mla).scatter_ref(want, slots)
        for a, b, c in zip(kv_a, kv_b, kv_c):
            for x, y, z in zip(*(t if isinstance(t, tuple) else (t,) for t in (a, b, c))):
                assert torch.equal(x, y), f"load call {call}"
                assert torch.equal(y, z), f"load call {call} vs the PyTorch oracle"


def test_noalloc_rejects_oversize():
    lib = _lib()
    cap = lib.lmc_noalloc_staging_capacity()
    kv = make_separate_kv(32, 64, 16, 8, 128, torch.bfloat16, DEV, seed=23)
    lay = PagedKVLayout(kv)
    T = 1024  # 32 layers x 2 x 1024 x 2 KiB = 128 MiB > capacity
    assert lay.chunk_bytes(T) > cap
    slots = block_slots(T, lay.block_size, lay.num_blocks, seed=33, device=DEV)
    host = torch.zeros(lay.chunk_shape(T), dtype=lay.dtype).pin_memory()
    rc, msg = _call(lib, lay, slots, host, True)
    assert rc == 3 and "exceeds" in msg
