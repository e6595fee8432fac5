"""TTFT-on-prefix-hit flow (tiny model on CPU; the same code times Qwen3-32B
on a B200 in bench.py)."""

import torch

from lmcache_ascend_b200.bench_ttft import run_ttft
from lmcache_ascend_b200.models.llama import LlamaConfig


def test_ttft_flow_cpu_tiny_model():
    mc = LlamaConfig(vocab_size=500, hidden_size=64, num_layers=3, num_heads=4,
                     num_kv_heads=2, head_dim=16, intermediate_size=96, max_position=2048,
                     qk_norm=True)
    r = run_ttft("cpu", tokens=600, requests=2, warmup=1, model_config=mc, chunk_size=256,
                 block_size=16, dtype=torch.float32)
    assert r["kv_check"] is True
    assert r["prefix_hit_tokens"] == 600
    assert r["p50_ms"] > 0
