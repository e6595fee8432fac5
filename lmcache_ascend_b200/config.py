"""Engine configuration: one dataclass, loaded from YAML, ``LMCACHE_*`` env
variables or a dict (vLLM ``kv_connector_extra_config``).

Key names follow upstream LMCache / the reference's extensions
(reference lmcache_ascend/__init__.py:78-310 adds the pd_*, p2p_*,
shared_cpu_cache_* and store_async* keys) so existing YAML files keep
working.  Keys of Ascend-only transports (hccl, hixl, hcomm) are accepted and
mapped onto the NVLink channel; see ``_ALIASES``.
"""

from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import yaml

from .utils.logging import init_logger

logger = init_logger(__name__)


def _size_gb(v: Any) -> float:
    return float(v)


@dataclass
class LMCacheEngineConfig:
    # --- chunking / engine ---------------------------------------------------
    chunk_size: int = 256
    save_unfull_chunk: bool = True
    hash_function: str = "xxh3_64"
    use_layerwise: bool = False
    store_async: bool = False
    store_async_max_queue_size: int = 64
    blocking_timeout_secs: float = 10.0
    # layerwise stores: bound on puts in flight to slower tiers
    layerwise_put_max_bytes: int = 4 << 30
    layerwise_put_max_batches: int = 64
    layerwise_put_timeout_secs: float = 60.0
    save_only_first_rank: bool = False  # MLA: replicated latent, rank 0 stores
    gpu_transfer_mode: str = "auto"     # auto | tma | simt
    cpu_transfer_mode: str = "copy_engine"  # copy_engine | zero_copy
    enable_nvtx: bool = False
    # --- local CPU ------------------------------------------------------------
    local_cpu: bool = True
    max_local_cpu_size: float = 5.0  # GB
    # HBM tier above the CPU tier (device-resident chunks, LRU with write-back
    # to the CPU tier on eviction)
    local_gpu: bool = False
    max_local_gpu_size: float = 0.0  # GB
    numa_node: int = -1  # >= 0: bind the CPU tier there, -1: no binding, -2: the GPU's node
    shared_cpu_cache: bool = False
    shared_cpu_cache_name: Optional[str] = None
    shared_cpu_cache_size: float = 0.0  # GB
    # --- local disk -----------------------------------------------------------
    local_disk: Optional[str] = None
    max_local_disk_size: float = 0.0  # GB
    # --- remote ---------------------------------------------------------------
    remote_url: Optional[str] = None
    remote_serde: str = "naive"  # naive | cachegen
    cachegen_k_bins: List[List[int]] = field(default_factory=lambda: [[0, 10, 32], [10, 10000, 16]])
    cachegen_v_bins: List[List[int]] = field(default_factory=lambda: [[0, 2, 32], [2, 10000, 16]])
    # --- CacheBlend -----------------------------------------------------------
    enable_blending: bool = False
    blend_recompute_ratios: List[float] = field(default_factory=lambda: [0.15])
    blend_check_layers: List[int] = field(default_factory=lambda: [1])
    blend_special_str: str = " # # "
    blend_min_tokens: int = 256
    # --- disaggregated prefill (PD) -------------------------------------------
    enable_pd: bool = False
    pd_role: Optional[str] = None  # sender | receiver
    transfer_channel: str = "nvlink"
    pd_buffer_size: int = 1 << 30
    pd_buffer_device: str = "cuda"
    pd_peer_host: Optional[str] = None
    pd_peer_init_port: List[int] = field(default_factory=lambda: [7300])
    pd_peer_alloc_port: List[int] = field(default_factory=lambda: [7400])
    pd_proxy_host: Optional[str] = None
    pd_proxy_port: Optional[int] = None
    pd_pull_mode: bool = False
    pd_delay_pull: bool = False
    pd_use_cpu_offload: bool = False
    pd_cpu_buffer_size: int = 0
    pd_alloc_fail_backoff_ttl: float = 5.0
    pd_pull_pending_ttl: float = 30.0
    pd_backpressure_reserve: float = 0.05
    pd_push_layerwise: bool = True
    pd_flag_timeout_s: float = 10.0
    # direct paged push: the decoder grants a push only into the slots it
    # reserved for the request (False: any in-range slots of a live, current
    # registration); the prefiller asks for the grant for at most this long
    pd_direct_require_reservation: bool = True
    pd_reserve_timeout_s: float = 5.0
    # --- P2P cross-instance ---------------------------------------------------
    enable_p2p: bool = False
    p2p_host: Optional[str] = None
    p2p_init_ports: List[int] = field(default_factory=lambda: [8200])
    p2p_lookup_ports: List[int] = field(default_factory=lambda: [8300])
    p2p_pull_pending_ttl: float = 30.0
    p2p_max_retries: int = 3
    controller_url: Optional[str] = None
    lmcache_instance_id: str = "lmcache_default_instance"
    # --- misc -----------------------------------------------------------------
    audit_actual_remove: bool = False
    enable_audit: bool = False
    enable_kv_events: bool = False
    extra_config: Dict[str, Any] = field(default_factory=dict)

    # --------------------------------------------------------------- loaders
    _ALIASES = {
        "max_local_cpu_size_gb": "max_local_cpu_size",
        "pd_transfer_channel": "transfer_channel",
    }
    _CHANNEL_ALIASES = {"hccl": "nvlink", "hixl": "nvlink", "hcomm_onesided": "nvlink",
                        "nixl": "nvlink"}

    @classmethod
    def field_names(cls) -> List[str]:
        return [f.name for f in dataclasses.fields(cls)]

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "LMCacheEngineConfig":
        cfg = cls()
        cfg.update(d)
        return cfg

    def update(self, d: Dict[str, Any]) -> "LMCacheEngineConfig":
        names = set(self.field_names())
        for k, v in (d or {}).items():
            k = k.removeprefix("lmcache.")
            k = self._ALIASES.get(k, k)
            if k not in names:
                self.extra_config[k] = v
                continue
            setattr(self, k, self._coerce(k, v))
        self.validate()
        return self

    @classmethod
    def from_file(cls, path: str) -> "LMCacheEngineConfig":
        with open(path) as f:
            d = yaml.safe_load(f) or {}
        return cls.from_dict(d)

    @classmethod
    def from_env(cls) -> "LMCacheEngineConfig":
        cfg = cls()
        path = os.environ.get("LMCACHE_CONFIG_FILE")
        if path:
            cfg = cls.from_file(path)
        env = {}
        for name in cls.field_names():
            v = os.environ.get("LMCACHE_" + name.upper())
            if v is not None:
                env[name] = v
        cfg.update(env)
        return cfg

    @classmethod
    def from_defaults(cls, **kw) -> "LMCacheEngineConfig":
        return cls.from_dict(kw)

    def _coerce(self, name: str, v: Any) -> Any:
        f = {f.name: f for f in dataclasses.fields(self)}[name]
        default = getattr(type(self)(), name)
        if v is None:
            return None
        typ = f.type if isinstance(f.type, str) else getattr(f.type, "__name__", "")
        if isinstance(v, str):
            s = v.strip()
            if "bool" in typ:
                return s.lower() in ("1", "true", "yes", "on")
            if typ in ("int",):
                return int(s)
            if typ in ("float",):
                return float(s)
            if "List" in typ or "Dict" in typ:
                try:
                    return json.loads(s)
                except json.JSONDecodeError:
                    return [type(default[0])(x) for x in s.split(",")] if default else s.split(",")
            return s
        if "List[int]" in typ and isinstance(v, int):
            return [v]
        return v

    def validate(self) -> None:
        if self.chunk_size <= 0:
            raise ValueError("chunk_size must be > 0")
        self.transfer_channel = self._CHANNEL_ALIASES.get(self.transfer_channel,
                                                          self.transfer_channel)
        if self.transfer_channel not in ("nvlink", "nccl", "tcp"):
            raise ValueError(f"unknown transfer_channel {self.transfer_channel!r}")
        if self.enable_pd and self.pd_role not in ("sender", "receiver"):
            raise ValueError("enable_pd requires pd_role 'sender' or 'receiver'")
        if self.remote_serde not in ("naive", "cachegen"):
            raise ValueError("remote_serde must be 'naive' or 'cachegen'")
        if self.gpu_transfer_mode not in ("auto", "tma", "simt"):
            raise ValueError("gpu_transfer_mode must be auto|tma|simt")
        if self.cpu_transfer_mode not in ("copy_engine", "zero_copy"):
            raise ValueError("cpu_transfer_mode must be copy_engine|zero_copy")
        if not (0.0 <= self.pd_backpressure_reserve < 1.0):
            raise ValueError("pd_backpressure_reserve must be in [0, 1)")

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


@dataclass
class LMCacheEngineMetadata:
    """Static facts about the model shard this engine serves."""

    model_name: str
    world_size: int
    worker_id: int
    fmt: str  # "vllm" | "sglang"
    kv_dtype: Any = None
    kv_shape: tuple = ()  # (num_layers, 2, chunk_size, num_kv_heads, head_size)
    use_mla: bool = False
    role: str = "worker"
    dp_rank: int = 0
    dp_size: int = 1
