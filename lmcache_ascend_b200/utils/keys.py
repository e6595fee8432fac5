"""Cache keys and deterministic token hashing.

A chunk key names one chunk of one KV shard:
``fmt@model@world_size@worker_id@hash@dtype[@group]`` -- the same fields as
upstream LMCache's ``CacheEngineKey`` (used throughout the reference, e.g.
lmcache_ascend/v1/token_database.py:94-110), so stores written by one
process can be found by another with the same model and parallel layout.

Token hashing chains chunks: ``h_i = H(h_{i-1}, tokens_i[, extra])``
(reference lmcache_ascend/v1/tokens_hash.py:9-30).  ``H`` must be identical in
every process; Python's builtin ``hash`` is only stable with
``PYTHONHASHSEED`` fixed, so the default here is xxh3-64 over the
little-endian int64 bytes of (prefix, tokens, extra).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple, Union

import hashlib
import numpy as np

try:  # xxhash is in the image; keep a pure fallback for other installs
    import xxhash

    def _xxh(data: bytes) -> int:
        return xxhash.xxh3_64_intdigest(data)
except Exception:  # pragma: no cover
    def _xxh(data: bytes) -> int:
        return int.from_bytes(hashlib.blake2b(data, digest_size=8).digest(), "little")

# Seed of the hash chain (the "prefix" of the first chunk).
NONE_HASH = 0x6C6D6361636865  # "lmcache"


def _tokens_bytes(tokens) -> bytes:
    if hasattr(tokens, "cpu") and hasattr(tokens, "numpy"):
        arr = tokens.detach().cpu().to(dtype=__import__("torch").int64).numpy()
    else:
        arr = np.asarray(tokens, dtype=np.int64)
    return np.ascontiguousarray(arr, dtype="<i8").tobytes()


def xxh3_hash_tokens(prefix_hash: Optional[int], tokens, extra: Any = None) -> int:
    p = NONE_HASH if prefix_hash is None else int(prefix_hash)
    data = (p & 0xFFFFFFFFFFFFFFFF).to_bytes(8, "little") + _tokens_bytes(tokens)
    if extra is not None:
        data += repr(extra).encode()
    return _xxh(data)


def sha256_hash_tokens(prefix_hash: Optional[int], tokens, extra: Any = None) -> int:
    p = NONE_HASH if prefix_hash is None else int(prefix_hash)
    h = hashlib.sha256((p & 0xFFFFFFFFFFFFFFFF).to_bytes(8, "little"))
    h.update(_tokens_bytes(tokens))
    if extra is not None:
        h.update(repr(extra).encode())
    return int.from_bytes(h.digest()[:8], "little")


def builtin_hash_tokens(prefix_hash: Optional[int], tokens, extra: Any = None) -> int:
    """Python ``hash`` of ``(prefix, tuple(tokens)[, extra])``; needs PYTHONHASHSEED."""
    if hasattr(tokens, "tolist"):
        tokens = tokens.tolist()
    if extra is None:
        return hash((prefix_hash, tuple(tokens))) & 0xFFFFFFFFFFFFFFFF
    return hash((prefix_hash, tuple(tokens), tuple(extra) if isinstance(extra, list) else extra)) \
        & 0xFFFFFFFFFFFFFFFF


HASH_FUNCTIONS: Dict[str, Callable[..., int]] = {
    "xxh3_64": xxh3_hash_tokens,
    "sha256": sha256_hash_tokens,
    "builtin": builtin_hash_tokens,
}


def get_hash_function(name: str) -> Callable[..., int]:
    try:
        return HASH_FUNCTIONS[name]
    except KeyError:
        raise ValueError(f"unknown hash function {name!r}; have {sorted(HASH_FUNCTIONS)}")


_KEY_FIELDS = ("fmt", "model_name", "world_size", "worker_id", "chunk_hash", "dtype", "group",
               "tags")


@dataclass(frozen=True, order=True)
class CacheEngineKey:
    fmt: str
    model_name: str
    world_size: int
    worker_id: int
    chunk_hash: int
    dtype: str = "bfloat16"
    group: int = 0  # KV layer group (0 regular/latent, 1 DSA indexer)
    tags: Tuple[Tuple[str, str], ...] = field(default=(), compare=True)

    # Keys are hashed and compared on every dict access of every tier (a
    # 16k-token layerwise request touches thousands of keys): the field tuple
    # and its hash are computed once per key, and equality compares the
    # cached tuples (the per-layer keys of one chunk share the same tuple).
    def __hash__(self) -> int:
        h = self.__dict__.get("_h")
        if h is None:
            h = hash(self._ft())
            object.__setattr__(self, "_h", h)
        return h

    def __eq__(self, other) -> bool:
        if self is other:
            return True
        if other.__class__ is not self.__class__:
            return NotImplemented
        a, b = self._ft(), other._ft()
        return a is b or a == b

    def _fields(self) -> tuple:
        return (self.fmt, self.model_name, self.world_size, self.worker_id, self.chunk_hash,
                self.dtype, self.group, self.tags)

    def _ft(self) -> tuple:
        t = self.__dict__.get("_t")
        if t is None:
            t = self._fields()
            object.__setattr__(self, "_t", t)
        return t

    # str hashes differ between processes: never ship the cached values
    def __getstate__(self) -> dict:
        d = dict(self.__dict__)
        d.pop("_h", None)
        d.pop("_t", None)
        return d

    def __setstate__(self, d: dict) -> None:
        for k, v in d.items():
            object.__setattr__(self, k, v)

    def to_string(self) -> str:
        s = (f"{self.fmt}@{self.model_name}@{self.world_size}@{self.worker_id}"
             f"@{self.chunk_hash:016x}@{self.dtype}")
        if self.group:
            s += f"@g{self.group}"
        for k, v in self.tags:
            s += f"@{k}%{v}"
        return s

    @staticmethod
    def from_string(s: str) -> "CacheEngineKey":
        parts = s.split("@")
        if len(parts) < 6:
            raise ValueError(f"invalid key string {s!r}")
        group, tags = 0, []
        for extra in parts[6:]:
            if extra.startswith("g") and extra[1:].isdigit():
                group = int(extra[1:])
            elif "%" in extra:
                k, v = extra.split("%", 1)
                tags.append((k, v))
        return CacheEngineKey(parts[0], parts[1], int(parts[2]), int(parts[3]),
                              int(parts[4], 16), parts[5], group, tuple(tags))

    @classmethod
    def create(cls, model_name: str, world_size: int, worker_id: int, chunk_hash: int,
               dtype: Any, tags: Optional[Dict[str, Any]] = None, kv_group: int = 0,
               fmt: str = "vllm") -> "CacheEngineKey":
        """Build a key from the argument order of upstream LMCache's
        ``CacheEngineKey(model_name, world_size, worker_id, chunk_hash, dtype,
        tags, kv_group=...)`` as the reference calls it (e.g. lmcache_ascend/
        v1/cache_engine.py:9854, tests/v1/test_shared_cpu_sparse_collective.py
        :178); ``dtype`` may be a torch dtype or its name."""
        name = str(dtype).removeprefix("torch.")
        tag_t = tuple(sorted((str(k), str(v)) for k, v in (tags or {}).items()))
        return cls(fmt, model_name, int(world_size), int(worker_id),
                   int(chunk_hash) & 0xFFFFFFFFFFFFFFFF, name, int(kv_group), tag_t)

    def with_worker(self, worker_id: int) -> "CacheEngineKey":
        return CacheEngineKey(self.fmt, self.model_name, self.world_size, worker_id,
                              self.chunk_hash, self.dtype, self.group, self.tags)

    def split_layers(self, num_layers: int) -> List["LayerCacheEngineKey"]:
        # bypasses the frozen-dataclass __init__ (one object.__setattr__ per
        # field): a layerwise request builds thousands of these.  Each layer
        # key shares this key's field tuple and gets its hash up front.
        base = {f: self.__dict__[f] for f in _KEY_FIELDS}
        base["_t"] = ft = self._ft()
        ph = hash(ft)
        out = []
        for i in range(num_layers):
            k = object.__new__(LayerCacheEngineKey)
            d = k.__dict__
            d.update(base)
            d["layer_id"] = i
            d["_h"] = hash((ph, i))
            out.append(k)
        return out

    def layer_key(self, layer_id: int) -> "LayerCacheEngineKey":
        k = object.__new__(LayerCacheEngineKey)
        d = k.__dict__
        d.update({f: self.__dict__[f] for f in _KEY_FIELDS})
        d["_t"] = ft = self._ft()
        d["layer_id"] = layer_id
        d["_h"] = hash((hash(ft), layer_id))
        return k

    def __str__(self) -> str:  # pragma: no cover - debugging aid
        return self.to_string()


@dataclass(frozen=True, order=True)
class LayerCacheEngineKey(CacheEngineKey):
    layer_id: int = 0

    def __hash__(self) -> int:
        h = self.__dict__.get("_h")
        if h is None:  # the value ``split_layers`` assigns
            h = hash((hash(self._ft()), self.layer_id))
            object.__setattr__(self, "_h", h)
        return h

    def __eq__(self, other) -> bool:
        if self is other:
            return True
        if other.__class__ is not self.__class__:
            return NotImplemented
        if self.layer_id != other.layer_id:
            return False
        a, b = self._ft(), other._ft()
        return a is b or a == b

    def to_string(self) -> str:
        return super().to_string() + f"@L{self.layer_id}"
