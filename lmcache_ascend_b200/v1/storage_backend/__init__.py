"""Storage backends and the factory that assembles the hierarchy.

Order (reference lmcache_ascend/v1/storage_backend/__init__.py:51-167):
PD -> [LocalGPU, the HBM tier this repo adds] -> LocalCPU -> P2P -> LocalDisk
-> Remote -> plugins, optionally wrapped by the audit backend.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Callable, Dict, Optional

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from ...utils.logging import init_logger
from .abstract_backend import StorageBackendInterface
from .local_cpu_backend import LocalCPUBackend

logger = init_logger(__name__)

# name -> factory(config, metadata, allocator_backend) for third-party tiers
PLUGIN_BACKENDS: Dict[str, Callable] = {}


def register_backend(name: str, factory: Callable) -> None:
    PLUGIN_BACKENDS[name] = factory


def CreateStorageBackends(config: LMCacheEngineConfig,
                          metadata: Optional[LMCacheEngineMetadata] = None,
                          dst_device: str = "cuda", **kw
                          ) -> "OrderedDict[str, StorageBackendInterface]":
    backends: "OrderedDict[str, StorageBackendInterface]" = OrderedDict()
    if config.enable_pd:
        from .pd.backend import PDBackend

        pd = PDBackend(config, metadata, **kw)
        backends[pd.name] = pd
    # The CPU tier always exists: it provides the allocator.  With
    # local_cpu=False it only allocates and does not keep objects.
    cpu = LocalCPUBackend(config, allocator=kw.get("cpu_allocator"))
    gpu = None
    if config.local_gpu and config.max_local_gpu_size > 0:
        from .local_gpu_backend import LocalGPUBackend

        gpu = LocalGPUBackend(config, lower=cpu)
        backends[gpu.name] = gpu  # first: it allocates the chunks of every store
    backends[cpu.name] = cpu
    if config.enable_p2p:
        from .p2p_backend import P2PBackend

        p2p = P2PBackend(config, metadata, cpu, hbm=gpu, **kw)
        backends[p2p.name] = p2p
    if config.local_disk:
        from .local_disk_backend import LocalDiskBackend

        disk = LocalDiskBackend(config, cpu)
        backends[disk.name] = disk
    if config.remote_url:
        from .remote_backend import RemoteBackend

        rb = RemoteBackend(config, metadata, cpu)
        backends[rb.name] = rb
    for name, factory in PLUGIN_BACKENDS.items():
        backends[name] = factory(config, metadata, cpu)
    if config.enable_audit:
        from .audit_backend import AuditBackend

        for name in list(backends):
            if name != cpu.name:
                backends[name] = AuditBackend(backends[name], config)
    return backends


__all__ = ["CreateStorageBackends", "LocalCPUBackend", "StorageBackendInterface",
           "register_backend"]
