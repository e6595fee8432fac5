"""Chunk key strings: layout, round trip, and keys built with the argument
order the reference uses for upstream LMCache's CacheEngineKey."""

import torch

from lmcache_ascend_b200.utils.keys import CacheEngineKey


def test_key_string_layout_and_round_trip():
    k = CacheEngineKey.create("model", 1, 0, 7, torch.float16)
    assert k.to_string() == "vllm@model@1@0@0000000000000007@float16"
    assert CacheEngineKey.from_string(k.to_string()) == k
    t = CacheEngineKey.create("Qwen3-32B", 4, 3, 0xDEADBEEF, torch.bfloat16,
                              {"lmcache.tag.internal.valid_tokens": 3}, kv_group=1)
    s = t.to_string()
    assert s == ("vllm@Qwen3-32B@4@3@00000000deadbeef@bfloat16@g1"
                 "@lmcache.tag.internal.valid_tokens%3")
    assert CacheEngineKey.from_string(s) == t
    # per-layer keys (layerwise stores) extend the chunk key
    lk = k.split_layers(2)
    assert [x.to_string() for x in lk] == [k.to_string() + "@L0", k.to_string() + "@L1"]
    assert lk[1] == k.layer_key(1) and hash(lk[1]) == hash(k.layer_key(1))
    # TP ranks differ only in the worker field; save_only_first_rank maps to 0
    assert k.with_worker(2).to_string() == "vllm@model@1@2@0000000000000007@float16"


def test_negative_hashes_wrap_to_64_bits():
    k = CacheEngineKey.create("m", 1, 0, -1, "float32")
    assert k.chunk_hash == 0xFFFFFFFFFFFFFFFF
    assert k.to_string().split("@")[4] == "ffffffffffffffff"
