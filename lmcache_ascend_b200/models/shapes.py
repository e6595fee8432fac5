"""KV-cache shapes of the model families the BASELINE configs name.

Used by the benchmarks, the tests and ``make_paged_cache`` to build
random-init paged caches of the right geometry (no checkpoints needed).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch


@dataclass(frozen=True)
class KVSpec:
    name: str
    num_layers: int
    num_kv_heads: int
    head_dim: int
    # MLA (DeepSeek): latent + rope widths instead of heads x head_dim
    kv_lora_rank: int = 0
    qk_rope_head_dim: int = 0
    indexer_dim: int = 0  # DSA lightning-indexer key width (int8 in C8 form)

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    def shard(self, tp: int) -> "KVSpec":
        """Per-rank shard: GQA heads split across TP ranks; MLA is replicated."""
        if self.is_mla:
            return self
        if self.num_kv_heads % tp:
            raise ValueError(f"{self.num_kv_heads} KV heads do not split over TP{tp}")
        return KVSpec(self.name + f"-tp{tp}", self.num_layers, self.num_kv_heads // tp,
                      self.head_dim)

    def token_bytes(self, dtype=torch.bfloat16) -> int:
        es = torch.empty((), dtype=dtype).element_size()
        if self.is_mla:
            return self.num_layers * (self.kv_lora_rank + self.qk_rope_head_dim) * es
        return self.num_layers * 2 * self.num_kv_heads * self.head_dim * es


LLAMA3_8B = KVSpec("Llama-3-8B", 32, 8, 128)
LLAMA31_8B = KVSpec("Llama-3.1-8B-Instruct", 32, 8, 128)
QWEN3_8B = KVSpec("Qwen3-8B", 36, 8, 128)
QWEN3_32B = KVSpec("Qwen3-32B", 64, 8, 128)
DEEPSEEK_V32 = KVSpec("DeepSeek-V3.2", 61, 1, 0, kv_lora_rank=512, qk_rope_head_dim=64,
                      indexer_dim=128)

SPECS = {s.name: s for s in (LLAMA3_8B, LLAMA31_8B, QWEN3_8B, QWEN3_32B, DEEPSEEK_V32)}


def make_paged_cache(spec: KVSpec, num_blocks: int, block_size: int,
                     dtype=torch.bfloat16, device="cuda", seed: int = 0,
                     layout: str = "separate") -> List:
    """Random-init paged cache in a vLLM layout.

    layout: ``separate`` -> per layer (K, V) [NB, BS, H, D];
    ``flash`` -> per layer [2, NB, BS, H, D]; MLA specs give per layer
    (k_nope [NB, BS, 1, r], k_pe [NB, BS, 1, rope]).
    """
    g = torch.Generator(device="cpu").manual_seed(seed)

    def rnd(*shape):
        return torch.randn(*shape, generator=g).to(dtype).to(device)

    out = []
    for _ in range(spec.num_layers):
        if spec.is_mla:
            out.append((rnd(num_blocks, block_size, 1, spec.kv_lora_rank),
                        rnd(num_blocks, block_size, 1, spec.qk_rope_head_dim)))
        elif layout == "flash":
            out.append(rnd(2, num_blocks, block_size, spec.num_kv_heads, spec.head_dim))
        else:
            out.append((rnd(num_blocks, block_size, spec.num_kv_heads, spec.head_dim),
                        rnd(num_blocks, block_size, spec.num_kv_heads, spec.head_dim)))
    return out


def block_table_slots(num_tokens: int, block_size: int, num_blocks: int, seed: int = 0,
                      device="cuda", dtype=torch.int32) -> torch.Tensor:
    """vLLM-like slot mapping: random block table, consecutive slots per block."""
    g = torch.Generator().manual_seed(seed)
    nblk = (num_tokens + block_size - 1) // block_size
    blocks = torch.randperm(num_blocks, generator=g)[:nblk]
    t = torch.arange(num_tokens)
    return (blocks[t // block_size] * block_size + t % block_size).to(dtype).to(device)
