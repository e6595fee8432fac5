"""Serialisers for the remote tier: ``naive`` (raw bytes + header) and
``cachegen`` (quantised + entropy coded, KV_2LTD chunks only).

Interface of upstream LMCache's serde (Serializer.serialize(memory_obj) ->
bytes object, Deserializer.deserialize(bytes) -> memory_obj), used by the
reference's remote backend with ``remote_serde`` (docs/cachegen/Cachegen.md).
"""

from __future__ import annotations

import json
import struct
from typing import Optional

import torch

from ...config import LMCacheEngineConfig
from ..cachegen import CacheGenConfig, CacheGenEncoded, decode_kv, decode_kv_bytes, encode_kv
from ..memory_management import MemoryFormat, MemoryObj

_NAIVE = b"LMCN"
_DTYPES = {str(d).removeprefix("torch."): d for d in
           (torch.float32, torch.float16, torch.bfloat16, torch.uint8, torch.int8)}


class NaiveSerde:
    name = "naive"

    def serialize(self, obj: MemoryObj) -> bytes:
        hdr = json.dumps({"shape": list(obj.get_shape()),
                          "dtype": str(obj.get_dtype()).removeprefix("torch."),
                          "fmt": obj.get_memory_format().name}).encode()
        n = obj.get_size()
        return _NAIVE + struct.pack("<I", len(hdr)) + hdr + \
            bytes(obj.raw_data[:n].cpu().numpy().tobytes())

    def deserialize(self, data: bytes, allocator) -> Optional[MemoryObj]:
        if data[:4] != _NAIVE:
            raise ValueError("not a naive-serde payload")
        (hl,) = struct.unpack("<I", data[4:8])
        hdr = json.loads(data[8:8 + hl])
        obj = allocator.allocate(torch.Size(hdr["shape"]), _DTYPES[hdr["dtype"]],
                                 MemoryFormat[hdr["fmt"]])
        if obj is None:
            return None
        payload = data[8 + hl:]
        obj.raw_data[:len(payload)].copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
        return obj


class CacheGenSerde:
    name = "cachegen"

    def __init__(self, config: LMCacheEngineConfig, num_layers: Optional[int] = None,
                 device: Optional[str] = None):
        self.config = config
        self.num_layers = num_layers
        self.device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self._cg: Optional[CacheGenConfig] = None

    def _cfg(self, L: int) -> CacheGenConfig:
        if self._cg is None or self._cg.nlayers != L:
            kr = [(a, min(b, L), c) for a, b, c in self.config.cachegen_k_bins if a < L]
            vr = [(a, min(b, L), c) for a, b, c in self.config.cachegen_v_bins if a < L]
            self._cg = CacheGenConfig.from_ranges(L, kr, vr)
        return self._cg

    def serialize(self, obj: MemoryObj) -> bytes:
        if obj.get_memory_format() != MemoryFormat.KV_2LTD:
            raise ValueError("CacheGen serde handles KV_2LTD chunks")
        kv = obj.tensor
        if self.device.startswith("cuda") and not kv.is_cuda:
            kv = kv.to(self.device, non_blocking=True)
        return encode_kv(kv, self._cfg(kv.shape[1])).to_bytes()

    def deserialize(self, data: bytes, allocator) -> Optional[MemoryObj]:
        L, T, C, dtype = CacheGenEncoded.peek_shape(data)
        obj = allocator.allocate(torch.Size([2, L, T, C]), dtype, MemoryFormat.KV_2LTD)
        if obj is None:
            return None
        if self.device.startswith("cuda"):
            # one H2D of the payload; the dequantise writes straight into a
            # device-resident object (else one copy into the host object)
            decode_kv_bytes(data, self.device, out=obj.tensor)
        else:
            obj.tensor.copy_(decode_kv(CacheGenEncoded.from_bytes(data), self.device))
        return obj


def create_serde(config: LMCacheEngineConfig):
    if config.remote_serde == "cachegen":
        return CacheGenSerde(config)
    return NaiveSerde()
