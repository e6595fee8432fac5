"""NVTX ranges for profiling (reference: ``_lmcache_nvtx_annotate``,
lmcache_ascend/v1/cache_engine.py:36).  Enabled with LMCACHE_NVTX=1; when
off, the decorator returns the function unchanged."""

from __future__ import annotations

import functools
import os

import torch

ENABLED = os.environ.get("LMCACHE_NVTX", "0") == "1"


def nvtx_range(name: str):
    def deco(fn):
        if not ENABLED:
            return fn

        @functools.wraps(fn)
        def wrapper(*a, **kw):
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*a, **kw)
            finally:
                torch.cuda.nvtx.range_pop()

        return wrapper

    return deco
