"""GPU connectors: paged KV cache <-> chunk objects.

Factory mirrors reference lmcache_ascend/v1/npu_connector/__init__.py:35-130
(pick by serving engine, layerwise, blending).
"""

from __future__ import annotations

from typing import Optional

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from .connector import (
    GPUConnectorInterface,
    SGLangGPUConnector,
    SGLangLayerwiseGPUConnector,
    VLLMBufferLayerwiseGPUConnector,
    VLLMPagedMemGPUConnector,
    VLLMPagedMemLayerwiseGPUConnector,
)


def CreateGPUConnector(config: LMCacheEngineConfig,
                       metadata: Optional[LMCacheEngineMetadata] = None,
                       engine: str = "vllm", device=None) -> GPUConnectorInterface:
    use_mla = bool(metadata.use_mla) if metadata is not None else False
    if engine == "sglang":
        if config.use_layerwise:
            return SGLangLayerwiseGPUConnector(config, device=device, use_mla=use_mla)
        return SGLangGPUConnector(config, device=device, use_mla=use_mla)
    if config.enable_blending:
        return VLLMBufferLayerwiseGPUConnector(config, device=device, use_mla=use_mla)
    if config.use_layerwise:
        return VLLMPagedMemLayerwiseGPUConnector(config, device=device, use_mla=use_mla)
    return VLLMPagedMemGPUConnector(config, device=device, use_mla=use_mla)


__all__ = [
    "CreateGPUConnector",
    "GPUConnectorInterface",
    "SGLangGPUConnector",
    "SGLangLayerwiseGPUConnector",
    "VLLMBufferLayerwiseGPUConnector",
    "VLLMPagedMemGPUConnector",
    "VLLMPagedMemLayerwiseGPUConnector",
]
