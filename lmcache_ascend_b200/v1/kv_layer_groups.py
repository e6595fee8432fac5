"""KV layer groups: layers whose caches share a storage shape and dtype.

A model's layers can differ in cache shape (hybrid attention, MLA latent vs
the DSA indexer, mixed int8/bf16 indexer precision) and dtype.  Grouping
them lets each group move with one paged layout and one kernel launch.
Behaviour of the reference (lmcache_ascend/v1/kv_layer_groups.py:97-181 and
the hidden-size rules at :73-94):

* a group key is the tuple of plane shapes and dtypes of one layer's cache;
* a tuple cache stores its planes concatenated along the hidden dimension
  (MLA/DSA), unless it is a (K, V) pair of equal shapes;
* an (int8 keys [NB, 128, 1, D], fp16 scales [NB, 128, 1, 1]) pair is a C8
  indexer cache stored as uint8 rows of D + 2 bytes per token;
* with a mixed-precision indexer policy every indexer layer joins one group
  whose rows are sized for the widest layer, and the registered dtypes must
  agree with the policy;
* groups are ordered by their first layer.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Set, Tuple, Union

import torch

from ..utils.logging import init_logger

logger = init_logger(__name__)

Cache = Union[torch.Tensor, Tuple[torch.Tensor, ...]]


@dataclass
class IndexerC8Policy:
    """Which indexer layers hold int8 keys + fp16 scales (C8) and which hold
    floating keys.  ``mixed`` = some of each."""

    key_dim: int = 128
    c8_layers: Set[int] = field(default_factory=set)
    num_indexer_layers: int = 0

    @property
    def token_bytes(self) -> int:
        return self.key_dim + 2  # int8 key bytes + one fp16 scale

    @property
    def mixed(self) -> bool:
        return 0 < len(self.c8_layers) < self.num_indexer_layers

    def is_c8(self, indexer_layer: int) -> bool:
        return indexer_layer in self.c8_layers


@dataclass
class KVLayerGroupInfo:
    layer_names: List[str]
    layer_indices: List[int]
    shape: torch.Size  # per-layer storage shape
    dtype: torch.dtype
    planes: int = 1

    @property
    def num_layers(self) -> int:
        return len(self.layer_indices)

    @property
    def hidden_dim_size(self) -> int:
        """Elements per token of one layer: H * D for [2, NB, BS, H, D] and
        [NB, BS, H, D], E for [NB, BS, E]."""
        s = self.shape
        if len(s) == 5:
            return int(s[3] * s[4])
        if len(s) == 4:
            if s[0] == 1:
                raise ValueError(f"invalid per-layer cache shape {tuple(s)}")
            return int(s[2] * s[3])
        if len(s) == 3:
            return int(s[2])
        raise ValueError(f"invalid per-layer cache shape {tuple(s)}")


def _tuple_storage_shape(planes: Sequence[torch.Tensor]) -> torch.Size:
    first = planes[0].shape
    for p in planes[1:]:
        if p.shape[:2] != first[:2]:
            raise ValueError("every plane of a layer must share [num_blocks, block_size], "
                             f"got {tuple(first)} and {tuple(p.shape)}")
    if len(planes) == 2 and planes[0].shape == planes[1].shape:
        return first
    hidden = sum(int(p.shape[-2] * p.shape[-1]) if p.dim() == 4 else int(p.shape[-1])
                 for p in planes)
    return torch.Size([first[0], first[1], hidden])


def group_key(cache: Cache) -> Tuple[tuple, torch.Size, torch.dtype, int]:
    """(grouping key, storage shape, storage dtype, planes) of one layer."""
    if isinstance(cache, torch.Tensor):
        return ((tuple(cache.shape),), (cache.dtype,)), cache.shape, cache.dtype, 1
    if not isinstance(cache, (tuple, list)) or not cache:
        raise TypeError(f"unknown KV cache type {type(cache)}")
    planes = tuple(cache)
    dtypes = tuple(p.dtype for p in planes)
    shapes = tuple(tuple(p.shape) for p in planes)
    if dtypes == (torch.int8, torch.float16):
        key, scale = planes
        if key.dim() != 4 or tuple(key.shape[1:3]) != (128, 1) or \
                tuple(scale.shape) != (*key.shape[:3], 1):
            raise ValueError("C8 indexer caches need keys [NB, 128, 1, D] and scales "
                             "[NB, 128, 1, 1]")
        return (shapes, dtypes), torch.Size([key.shape[0], key.shape[1], key.shape[-1] + 2]), \
            torch.uint8, 2
    if len(set(dtypes)) != 1:
        raise ValueError("a layer's planes must share one dtype (C8 indexer excepted)")
    return (shapes, dtypes), _tuple_storage_shape(planes), dtypes[0], len(planes)


class KVLayerGroupsManager:
    def __init__(self) -> None:
        self.kv_layer_groups: List[KVLayerGroupInfo] = []
        self._group_of: Dict[int, int] = {}

    def build_kv_layer_groups(self, kv_caches: "Dict[str, Cache]",
                              indexer_policy: Optional[IndexerC8Policy] = None) -> None:
        """Group ``{layer_name: cache}`` (model order).  No-op once built."""
        if self.kv_layer_groups or not kv_caches:
            return
        members: "OrderedDict[tuple, List[Tuple[str, int]]]" = OrderedDict()
        info: Dict[tuple, Tuple[torch.Size, torch.dtype, int]] = {}
        mixed = indexer_policy is not None and indexer_policy.mixed
        indexer_layer = 0
        for idx, (name, cache) in enumerate(kv_caches.items()):
            key, shape, dtype, planes = group_key(cache)
            if mixed and "indexer" in name:
                first = cache[0] if isinstance(cache, (tuple, list)) else cache
                if (first.dtype == torch.int8) != indexer_policy.is_c8(indexer_layer):
                    raise ValueError(f"indexer layer {name}: registered dtype {first.dtype} "
                                     "disagrees with the C8 policy")
                key = ("mixed_indexer",)
                # rows sized for the widest layer (bf16 keys: 2 bytes per element)
                width = max(indexer_policy.token_bytes, 2 * indexer_policy.key_dim)
                shape = torch.Size([first.shape[0], first.shape[1], width])
                dtype, planes = torch.uint8, 2
                indexer_layer += 1
            members.setdefault(key, []).append((name, idx))
            info[key] = (shape, dtype, planes)
        if mixed and indexer_layer != indexer_policy.num_indexer_layers:
            raise ValueError(f"{indexer_layer} indexer layers registered, policy names "
                             f"{indexer_policy.num_indexer_layers}")
        for key in sorted(members, key=lambda k: members[k][0][1]):
            names, idxs = zip(*members[key])
            shape, dtype, planes = info[key]
            self.kv_layer_groups.append(KVLayerGroupInfo(list(names), list(idxs), shape, dtype,
                                                         planes))
        for g, grp in enumerate(self.kv_layer_groups):
            for i in grp.layer_indices:
                self._group_of[i] = g
        logger.info("KV layer groups: %s", [(g.num_layers, tuple(g.shape), g.dtype)
                                             for g in self.kv_layer_groups])

    @property
    def num_groups(self) -> int:
        return len(self.kv_layer_groups)

    def group_of(self, layer_index: int) -> int:
        return self._group_of[layer_index]

    def caches_of(self, group: int, kv_caches: "Dict[str, Cache]") -> List[Cache]:
        """The caches of one group's layers, in layer order."""
        return [kv_caches[n] for n in self.kv_layer_groups[group].layer_names]

    def layouts(self, kv_caches: "Dict[str, Cache]", use_mla: bool = False):
        """One paged layout per group, so each group moves in one launch."""
        from .kv_format import PagedKVLayout

        return [PagedKVLayout(self.caches_of(g, kv_caches), use_mla=use_mla)
                for g in range(self.num_groups)]
