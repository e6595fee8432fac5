"""Token databases: map a token sequence to chunk keys.

``ChunkedTokenDatabase`` cuts the sequence into ``chunk_size`` chunks and
chains their hashes (a chunk's key depends on every token before it), so a
lookup finds the longest cached prefix.  ``SegmentTokenDatabase`` (CacheBlend)
splits on a separator token sequence and hashes every segment on its own, so
a document chunk is found wherever it appears in a prompt.

Semantics follow reference lmcache_ascend/v1/token_database.py:17-119
(``process_tokens``: mask prefix of Falses is skipped; hashes+offsets mode
for callers that already hold chunk hashes) and tokens_hash.py:9-30.
"""

from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from ..config import LMCacheEngineConfig, LMCacheEngineMetadata
from ..utils.keys import CacheEngineKey, NONE_HASH, get_hash_function
from ..utils.logging import init_logger

logger = init_logger(__name__)

ProcessTokensResult = Tuple[int, int, Union[CacheEngineKey, int]]
Tokens = Union[torch.Tensor, Sequence[int], np.ndarray]


def _to_numpy(tokens: Tokens) -> np.ndarray:
    if isinstance(tokens, torch.Tensor):
        return tokens.detach().cpu().to(torch.int64).numpy()
    return np.asarray(tokens, dtype=np.int64)


def _num_falses(mask: Optional[torch.Tensor], n: int) -> int:
    if mask is None:
        return 0
    m = mask.detach().cpu() if isinstance(mask, torch.Tensor) else torch.as_tensor(mask)
    return int(m.numel() - int(m.long().sum().item()))


class TokenDatabase:
    def __init__(self, config: Optional[LMCacheEngineConfig] = None,
                 metadata: Optional[LMCacheEngineMetadata] = None):
        self.config = config or LMCacheEngineConfig()
        self.metadata = metadata
        self.chunk_size = self.config.chunk_size
        self.save_unfull_chunk = self.config.save_unfull_chunk
        self.hash_func = get_hash_function(self.config.hash_function)

    # -------------------------------------------------------------- helpers
    def _hash_tokens(self, tokens, prefix_hash: Optional[int] = None,
                     extra_keys=None) -> int:
        return self.hash_func(prefix_hash, tokens, extra_keys)

    def _make_key_by_hash(self, chunk_hash: int, request_configs: Optional[dict] = None,
                          group: int = 0) -> CacheEngineKey:
        md = self.metadata
        tags = ()
        if request_configs:
            tags = tuple(sorted((str(k).removeprefix("lmcache.tag."), str(v))
                                for k, v in request_configs.items()
                                if str(k).startswith("lmcache.tag.")))
        if md is None:
            return CacheEngineKey("vllm", "model", 1, 0, chunk_hash, "bfloat16", group, tags)
        dtype = str(md.kv_dtype).removeprefix("torch.") if md.kv_dtype is not None else "bfloat16"
        return CacheEngineKey(md.fmt, md.model_name, md.world_size, md.worker_id,
                              chunk_hash, dtype, group, tags)

    def process_tokens(self, tokens: Optional[Tokens] = None,
                       hashes: Optional[List[int]] = None,
                       offsets: Optional[List[int]] = None,
                       mask: Optional[torch.Tensor] = None, make_key: bool = True,
                       request_configs: Optional[dict] = None
                       ) -> Iterable[ProcessTokensResult]:
        raise NotImplementedError


class ChunkedTokenDatabase(TokenDatabase):
    """Prefix-chained fixed-size chunks."""

    def chunk_hashes(self, tokens: Tokens, extra_keys=None) -> List[int]:
        arr = _to_numpy(tokens)
        out, prefix = [], None
        n = len(arr)
        for start in range(0, n, self.chunk_size):
            end = min(start + self.chunk_size, n)
            if end - start < self.chunk_size and not self.save_unfull_chunk:
                break
            prefix = self._hash_tokens(arr[start:end], prefix if prefix is not None else NONE_HASH,
                                       extra_keys)
            out.append(prefix)
        return out

    def process_tokens(self, tokens: Optional[Tokens] = None,
                       hashes: Optional[List[int]] = None,
                       offsets: Optional[List[int]] = None,
                       mask: Optional[torch.Tensor] = None, make_key: bool = True,
                       request_configs: Optional[dict] = None
                       ) -> Iterable[ProcessTokensResult]:
        if tokens is not None:
            arr = _to_numpy(tokens)
            n = len(arr)
            if n == 0:
                return
            nf = _num_falses(mask, n)
            if nf >= n:
                return
            if nf % self.chunk_size != 0:
                raise ValueError(
                    f"masked prefix ({nf}) must be a multiple of chunk_size ({self.chunk_size})")
            prefix = None
            for start in range(0, n, self.chunk_size):
                end = min(start + self.chunk_size, n)
                if end - start < self.chunk_size and not self.save_unfull_chunk:
                    return
                prefix = self._hash_tokens(arr[start:end], NONE_HASH if prefix is None else prefix)
                if start < nf:
                    continue
                yield (start, end,
                       self._make_key_by_hash(prefix, request_configs) if make_key else prefix)
        elif hashes is not None:
            if offsets is None:
                raise ValueError("If hashes are provided, offsets must also be provided.")
            start = 0
            for h, off in zip(hashes, offsets):
                end = start + off
                yield (start, end, self._make_key_by_hash(h, request_configs) if make_key else h)
                start = end
        else:
            raise ValueError("Either tokens or hashes must be provided.")


class SegmentTokenDatabase(TokenDatabase):
    """Separator-split segments, each hashed independently (CacheBlend)."""

    def __init__(self, config: Optional[LMCacheEngineConfig] = None,
                 metadata: Optional[LMCacheEngineMetadata] = None,
                 sep_tokens: Optional[Sequence[int]] = None):
        super().__init__(config, metadata)
        self.sep_tokens = np.asarray(list(sep_tokens or []), dtype=np.int64)
        self.sep_len = len(self.sep_tokens)

    def _fast_split_by_subtensor(self, arr: np.ndarray) -> List[np.ndarray]:
        if self.sep_len == 0:
            return [arr]
        n, k = len(arr), self.sep_len
        if n < k:
            return [arr]
        win = np.lib.stride_tricks.sliding_window_view(arr, k)
        hits = np.nonzero((win == self.sep_tokens).all(axis=1))[0]
        parts, start = [], 0
        last_end = -1
        for h in hits:
            if h < last_end:
                continue  # overlapping match
            parts.append(arr[start:h])
            start = h + k
            last_end = start
        parts.append(arr[start:])
        return parts

    def process_tokens(self, tokens: Optional[Tokens] = None,
                       hashes: Optional[List[int]] = None,
                       offsets: Optional[List[int]] = None,
                       mask: Optional[torch.Tensor] = None, make_key: bool = True,
                       request_configs: Optional[dict] = None
                       ) -> Iterable[ProcessTokensResult]:
        if tokens is None:
            if hashes is None:
                raise ValueError("Either tokens or hashes must be provided.")
            yield from ChunkedTokenDatabase.process_tokens(self, None, hashes, offsets,
                                                           mask, make_key, request_configs)
            return
        arr = _to_numpy(tokens)
        n = len(arr)
        if n == 0:
            logger.warning("process_tokens: empty token list")
            return
        nf = _num_falses(mask, n)
        if nf >= n:
            return
        start = 0
        for i, seg in enumerate(self._fast_split_by_subtensor(arr)):
            if i > 0:
                start += self.sep_len
            end = start + len(seg)
            if start >= nf and len(seg) > 0:
                h = self._hash_tokens(seg)
                yield (start, end, self._make_key_by_hash(h, request_configs) if make_key else h)
            start = end
