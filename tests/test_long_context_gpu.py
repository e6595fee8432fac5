"""Long-context qualification: one 512k-token request through the engine.

Llama-3-8B-shaped KV rows (8 KV heads x 128, bf16: 2 KB per token and
plane), 2 layers, block size 128.  The paged planes are just over 2 GiB each, so slot
byte offsets pass 2^31: any 32-bit offset arithmetic on the store or the
retrieve path shows up as wrong rows.  The prefix is stored from one set of
blocks into the HBM tier (2048 chunks of 256 tokens), looked up, and
retrieved into a disjoint set of blocks taken from the top half of the
cache; every row is compared.  Checked on a B200: 8 GiB of paged cache plus
4 GiB of HBM tier.
"""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

pytestmark = pytest.mark.gpu

T = 512 * 1024
L, H, D, BS = 2, 8, 128, 128
NB = 2 * T // BS + 64  # the top blocks' rows start past 2^31 bytes


def _slots(blocks: torch.Tensor) -> torch.Tensor:
    t = torch.arange(T, device=blocks.device)
    return blocks[t // BS] * BS + t % BS


def test_512k_token_prefix_store_lookup_retrieve():
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    kv = [(torch.randn(NB, BS, H, D, device=dev, generator=g).to(torch.bfloat16),
           torch.randn(NB, BS, H, D, device=dev, generator=g).to(torch.bfloat16))
          for _ in range(L)]
    kv_bytes = T * L * 2 * H * D * 2
    cfg = LMCacheEngineConfig.from_defaults(
        chunk_size=256, local_gpu=True, max_local_gpu_size=kv_bytes * 1.02 / (1 << 30),
        max_local_cpu_size=0.05)
    md = LMCacheEngineMetadata("llama3-8b-shape", 1, 0, "vllm", torch.bfloat16)
    eng = LMCacheEngine(cfg, md, VLLMPagedMemGPUConnector(cfg, kvcaches=kv))
    try:
        perm = torch.randperm(NB, device=dev, generator=g)
        # source blocks from the lower half, destination blocks from the upper
        # half of the cache: destination offsets are past 2^31 bytes
        lower = perm[perm < NB // 2][: T // BS]
        upper = perm[perm >= NB // 2][: T // BS]
        src = _slots(lower)
        dst = _slots(upper)
        assert int(dst.max()) * H * D * 2 >= 2 ** 31
        tokens = torch.randint(0, 128000, (T,), generator=torch.Generator().manual_seed(1))
        eng.store(tokens, slot_mapping=src)
        torch.cuda.synchronize()
        assert eng.lookup(tokens) == T
        ret = eng.retrieve(tokens, slot_mapping=dst)
        torch.cuda.synchronize()
        assert int(ret.sum()) == T
        for k, v in kv:
            for plane in (k, v):
                rows = plane.view(NB * BS, H * D)
                assert torch.equal(rows[src], rows[dst])
    finally:
        eng.close()
