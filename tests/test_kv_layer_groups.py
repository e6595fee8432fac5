"""KV layer groups (reference lmcache_ascend/v1/kv_layer_groups.py behaviour)."""

import pytest
import torch

from lmcache_ascend_b200.v1.kv_layer_groups import (IndexerC8Policy, KVLayerGroupInfo,
                                                    KVLayerGroupsManager, group_key)


def test_uniform_layers_one_group_and_hidden_size():
    caches = {f"model.layers.{i}.attn": (torch.zeros(4, 16, 2, 64), torch.zeros(4, 16, 2, 64))
              for i in range(3)}
    m = KVLayerGroupsManager()
    m.build_kv_layer_groups(caches)
    assert m.num_groups == 1
    g = m.kv_layer_groups[0]
    assert g.layer_indices == [0, 1, 2] and g.hidden_dim_size == 128 and g.dtype == torch.float32
    assert len(m.layouts(caches)) == 1
    m.build_kv_layer_groups({"x": torch.zeros(1)})  # already built: no-op
    assert m.num_groups == 1


def test_mixed_shapes_split_in_layer_order():
    a = (torch.zeros(4, 16, 2, 64), torch.zeros(4, 16, 2, 64))
    b = (torch.zeros(4, 16, 1, 128), torch.zeros(4, 16, 1, 128))
    caches = {"l.0": b, "l.1": a, "l.2": b, "l.3": a}
    m = KVLayerGroupsManager()
    m.build_kv_layer_groups(caches)
    assert [g.layer_indices for g in m.kv_layer_groups] == [[0, 2], [1, 3]]
    assert m.group_of(3) == 1
    assert [len(c) for c in (m.caches_of(0, caches), m.caches_of(1, caches))] == [2, 2]


def test_mla_tuple_concatenates_hidden_and_c8_rows():
    mla = (torch.zeros(8, 64, 1, 512, dtype=torch.bfloat16),
           torch.zeros(8, 64, 1, 64, dtype=torch.bfloat16))
    key, shape, dtype, planes = group_key(mla)
    assert tuple(shape) == (8, 64, 576) and planes == 2
    c8 = (torch.zeros(8, 128, 1, 128, dtype=torch.int8),
          torch.zeros(8, 128, 1, 1, dtype=torch.float16))
    _, shape, dtype, _ = group_key(c8)
    assert tuple(shape) == (8, 128, 130) and dtype == torch.uint8
    with pytest.raises(ValueError):
        group_key((torch.zeros(8, 128, 1, 128, dtype=torch.int8),
                   torch.zeros(8, 64, 1, 1, dtype=torch.float16)))
    with pytest.raises(ValueError):
        group_key((torch.zeros(4, 16, 8), torch.zeros(4, 16, 8, dtype=torch.float16)))
    assert KVLayerGroupInfo(["a"], [0], torch.Size([8, 64, 576]), torch.bfloat16).hidden_dim_size \
        == 576


def test_mixed_indexer_policy_groups_and_validates():
    c8 = (torch.zeros(8, 128, 1, 128, dtype=torch.int8),
          torch.zeros(8, 128, 1, 1, dtype=torch.float16))
    fp = torch.zeros(8, 128, 1, 128, dtype=torch.bfloat16)
    lat = torch.zeros(8, 128, 576, dtype=torch.bfloat16)
    caches = {"l.0.attn": lat, "l.0.indexer": c8, "l.1.attn": lat, "l.1.indexer": fp}
    pol = IndexerC8Policy(128, {0}, 2)
    assert pol.mixed and pol.token_bytes == 130
    m = KVLayerGroupsManager()
    m.build_kv_layer_groups(caches, pol)
    assert [g.layer_names for g in m.kv_layer_groups] == [["l.0.attn", "l.1.attn"],
                                                         ["l.0.indexer", "l.1.indexer"]]
    assert m.kv_layer_groups[1].dtype == torch.uint8 and m.kv_layer_groups[1].shape[2] == 256
    with pytest.raises(ValueError):  # dtype disagrees with policy
        KVLayerGroupsManager().build_kv_layer_groups(caches, IndexerC8Policy(128, {1}, 2))
    with pytest.raises(ValueError):  # layer count disagrees with policy
        KVLayerGroupsManager().build_kv_layer_groups(caches, IndexerC8Policy(128, {0}, 3))
