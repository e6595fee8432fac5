"""vLLM v1 KV connector class (``KVConnectorBase_V1``) backed by this engine.

Use from vLLM:
    KVTransferConfig(kv_connector="LMCacheB200ConnectorV1",
                     kv_connector_module_path=
                         "lmcache_ascend_b200.integration.vllm.connector",
                     kv_role="kv_both",
                     kv_connector_extra_config={"lmcache.chunk_size": 256, ...})

Counterpart of the reference's ``LMCacheAscendConnectorV1Dynamic``
(lmcache_ascend/integration/vllm/lmcache_ascend_connector_v1.py:34-217):
the DP rank/size of vLLM's parallel config are folded into the engine
metadata, ``lmcache.*`` extra-config keys override the engine config, and
all logic lives in ``adapter.LMCacheConnectorV1Impl``.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
)

from .adapter import LMCacheConnectorMetadata, LMCacheConnectorV1Impl, config_from_extra


class LMCacheB200ConnectorMetadata(KVConnectorMetadata, LMCacheConnectorMetadata):
    pass


class LMCacheB200ConnectorV1(KVConnectorBase_V1):
    def __init__(self, vllm_config, role: KVConnectorRole, kv_cache_config=None):
        super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
        kvt = vllm_config.kv_transfer_config
        extra = dict(kvt.kv_connector_extra_config or {}) if kvt is not None else {}
        cfg = config_from_extra(extra)
        pc = vllm_config.parallel_config
        mc = vllm_config.model_config
        r = "scheduler" if role == KVConnectorRole.SCHEDULER else "worker"
        tp_rank = 0
        if r == "worker":
            try:
                from vllm.distributed.parallel_state import get_tensor_model_parallel_rank

                tp_rank = get_tensor_model_parallel_rank()
            except Exception:
                tp_rank = 0
        self._impl = LMCacheConnectorV1Impl(
            r, cfg, model_name=str(mc.model), block_size=vllm_config.cache_config.block_size,
            world_size=pc.tensor_parallel_size, rank=tp_rank, use_mla=bool(mc.use_mla),
            dp_rank=getattr(pc, "data_parallel_rank", 0) or 0, kv_dtype=None,
            kv_role=getattr(kvt, "kv_role", None) or "kv_both")

    # ---------------------------------------------------------- worker
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self._impl.register_kv_caches(kv_caches)

    def bind_connector_metadata(self, connector_metadata: KVConnectorMetadata) -> None:
        super().bind_connector_metadata(connector_metadata)
        self._impl.bind_connector_metadata(connector_metadata)

    def clear_connector_metadata(self) -> None:
        super().clear_connector_metadata()
        self._impl.clear_connector_metadata()

    def handle_preemptions(self, kv_connector_metadata: KVConnectorMetadata):
        self._impl.handle_preemptions(kv_connector_metadata)

    def on_new_request(self, request):
        self._impl.on_new_request(request)

    def start_load_kv(self, forward_context, **kwargs: Any) -> None:
        self._impl.start_load_kv(forward_context, **kwargs)

    def wait_for_layer_load(self, layer_name: str) -> None:
        self._impl.wait_for_layer_load(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata,
                      **kwargs: Any) -> None:
        self._impl.save_kv_layer(layer_name, kv_layer, attn_metadata, **kwargs)

    def wait_for_save(self):
        self._impl.wait_for_save()

    def get_finished(self, finished_req_ids: set[str]):
        return self._impl.get_finished(finished_req_ids)

    def get_block_ids_with_load_errors(self) -> set[int]:
        return self._impl.get_block_ids_with_load_errors()

    # ------------------------------------------------------- scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        return self._impl.get_num_new_matched_tokens(request, num_computed_tokens)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        self._impl.update_state_after_alloc(request, blocks, num_external_tokens)

    def build_connector_meta(self, scheduler_output) -> KVConnectorMetadata:
        m = self._impl.build_connector_meta(scheduler_output)
        out = LMCacheB200ConnectorMetadata()
        out.requests = m.requests
        out.preemption_captures = m.preemption_captures
        out.preemption_cancels = m.preemption_cancels
        return out

    def request_finished(self, request, block_ids: list[int]):
        return self._impl.request_finished(request, block_ids)

    def shutdown(self):
        self._impl.shutdown()
