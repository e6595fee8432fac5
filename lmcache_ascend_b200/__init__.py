"""lmcache_ascend_b200: a KV-cache engine for NVIDIA B200 (sm_100a).

Token-hash chunked KV store/retrieve/lookup over pinned-CPU, local-disk and
remote tiers; a vLLM v1 / SGLang connector; disaggregated prefill with a fused
NVLink push kernel; CacheGen compression and CacheBlend re-positioning.
Feature parity target: LMCache-Ascend (qiuziyan1998/LMCache-Ascend).
"""

__version__ = "0.1.0"

from .config import LMCacheEngineConfig, LMCacheEngineMetadata  # noqa: E402

__all__ = ["LMCacheEngineConfig", "LMCacheEngineMetadata", "__version__"]
