"""Page-window planning (reference lmcache_ascend/v1/direct_store_plan.py:23-129):
a request's tokens are placed in windows of whole blocks, at most
``window_tokens`` per window (rounded down to whole blocks, at least one
block); the last window holds the remainder."""

from __future__ import annotations

from typing import List, Tuple


def plan_windows(num_tokens: int, block_size: int, window_tokens: int) -> List[Tuple[int, int]]:
    if num_tokens <= 0:
        return []
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    w = max(block_size, (max(window_tokens, 1) // block_size) * block_size)
    return [(s, min(num_tokens, s + w)) for s in range(0, num_tokens, w)]
