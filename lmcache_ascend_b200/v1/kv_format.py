"""KV-cache format detection and the paged-layout descriptor.

``KVCacheFormat`` and ``detect`` keep the reference's format vocabulary and
detection rules (reference lmcache_ascend/v1/kv_format.py:13-219) so callers
can pass the same ``kvcaches`` structures.  ``MLA_FLAT`` is added for vLLM's
CUDA MLA cache, one ``[num_blocks, block_size, kv_lora_rank + rope_dim]``
tensor per layer.

``PagedKVLayout`` reduces any format to planes (K, V, k_nope, k_pe, indexer)
with per-plane block/slot strides and row sizes.  The same description drives
the CUDA kernels (``PagedLayout`` in the native module) and the PyTorch
oracle used on CPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import List, Optional, Sequence, Tuple, Union

import torch

from ..utils.logging import init_logger

logger = init_logger(__name__)

KVCaches = Sequence[Union[torch.Tensor, Tuple[torch.Tensor, ...]]]


class KVCacheFormat(Enum):
    UNDEFINED = 0
    MERGED_KV = 1    # layer: [2, NB, BS, H, D] (flash) or [NB, 2, BS, H, D] (flashinfer)
    SEPARATE_KV = 2  # layer: (K, V) each [NB, BS, H, D]; SGLang: [K_all, V_all] 5-D
    MLA_KV = 3       # layer: (k_nope [NB, BS, 1, Dk], k_pe [NB, BS, 1, Dr])
    DSA_KV = 4       # layer: (k_nope, k_pe, indexer_k [NB, BS, 1, Di])
    MLA_LATENT = 5   # two-group DSA path, latent group: (k_nope, k_pe)
    DSA_INDEX = 6    # two-group DSA path, indexer group: (indexer_k,)
    MLA_FLAT = 7     # vLLM CUDA MLA: layer: [NB, BS, Dk + Dr]

    def is_separate_format(self) -> bool:
        return self == KVCacheFormat.SEPARATE_KV

    def is_merged_format(self) -> bool:
        return self == KVCacheFormat.MERGED_KV

    def is_mla_format(self) -> bool:
        return self in (KVCacheFormat.MLA_KV, KVCacheFormat.MLA_LATENT, KVCacheFormat.MLA_FLAT)

    def is_mla_latent_format(self) -> bool:
        return self == KVCacheFormat.MLA_LATENT

    def is_dsa_format(self) -> bool:
        return self in (KVCacheFormat.DSA_KV, KVCacheFormat.DSA_INDEX)

    def is_dsa_index_format(self) -> bool:
        return self == KVCacheFormat.DSA_INDEX

    def is_tuple_format(self) -> bool:
        return self in (
            KVCacheFormat.SEPARATE_KV,
            KVCacheFormat.MLA_KV,
            KVCacheFormat.DSA_KV,
            KVCacheFormat.MLA_LATENT,
            KVCacheFormat.DSA_INDEX,
        )

    def get_kv_size(self) -> int:
        if self == KVCacheFormat.DSA_KV:
            return 3
        if self in (KVCacheFormat.SEPARATE_KV, KVCacheFormat.MLA_KV, KVCacheFormat.MLA_LATENT):
            return 2
        if self in (KVCacheFormat.MERGED_KV, KVCacheFormat.DSA_INDEX, KVCacheFormat.MLA_FLAT):
            return 1
        return 0

    @property
    def kv_group(self) -> int:
        """0 = latent/regular group, 1 = indexer group."""
        return 1 if self == KVCacheFormat.DSA_INDEX else 0

    @property
    def uses_2ltd_chunks(self) -> bool:
        """True when chunks are ``[2, L, T, H*D]`` (KV_2LTD)."""
        return self in (KVCacheFormat.MERGED_KV, KVCacheFormat.SEPARATE_KV)

    @staticmethod
    def detect(kvcaches: KVCaches, use_mla: bool = False,
               dsa_two_groups: bool = False) -> "KVCacheFormat":
        """Detection rules of the reference (kv_format.py:131-219), plus MLA_FLAT."""
        if kvcaches is None or len(kvcaches) == 0:
            return KVCacheFormat.UNDEFINED
        first = kvcaches[0]
        if isinstance(kvcaches, list) and len(kvcaches) == 2:
            if isinstance(first, torch.Tensor) and first.ndim == 5 and first.shape[0] != 2 \
                    and first.shape[1] != 2:
                return KVCacheFormat.SEPARATE_KV
        if isinstance(first, tuple):
            n = len(first)
            if n == 3 and all(isinstance(t, torch.Tensor) for t in first):
                if first[0].shape != first[1].shape:
                    return KVCacheFormat.DSA_KV
            if n == 1 and dsa_two_groups and isinstance(first[0], torch.Tensor):
                return KVCacheFormat.DSA_INDEX
            if n == 2:
                k, v = first
                if isinstance(k, torch.Tensor) and isinstance(v, torch.Tensor):
                    if use_mla or k.shape != v.shape:
                        return KVCacheFormat.MLA_LATENT if dsa_two_groups else KVCacheFormat.MLA_KV
                    return KVCacheFormat.SEPARATE_KV
            return KVCacheFormat.SEPARATE_KV
        if isinstance(first, torch.Tensor):
            if first.ndim == 5 and (first.shape[0] == 2 or first.shape[1] == 2):
                return KVCacheFormat.MERGED_KV
            if first.ndim == 3 and use_mla:
                return KVCacheFormat.MLA_FLAT
        return KVCacheFormat.UNDEFINED


@dataclass
class Plane:
    """One component of a layer's paged cache.

    ``views`` per layer: [NB, BS, E] when a slot's row is contiguous, or
    [NB, BS, H, D] when the cache stores heads apart (head-major "HND"
    storage behind a token-major shape; vLLM uses it for some attention
    backends).  In the latter case a row is H segments of D elements,
    ``seg_stride`` elements apart.
    """

    views: List[torch.Tensor]
    row_elems: int
    elem_size: int
    seg_elems: int = 0   # 0: contiguous rows
    seg_stride: int = 0  # elements between a row's segments

    @property
    def row_bytes(self) -> int:
        return self.row_elems * self.elem_size

    @property
    def segmented(self) -> bool:
        return 0 < self.seg_elems < self.row_elems

    def rows(self, layer: int, blk, off) -> torch.Tensor:
        r = self.views[layer][blk, off]
        return r.reshape(r.shape[0], -1) if self.segmented else r

    def set_rows(self, layer: int, blk, off, rows: torch.Tensor) -> None:
        v = self.views[layer]
        v[blk, off] = rows.view(rows.shape[0], *v.shape[2:]) if self.segmented else rows


def _as_rows(t: torch.Tensor):
    """[NB, BS, ...] -> (view, seg_elems, seg_stride): a contiguous [NB, BS, E]
    row view, or the [NB, BS, H, D] tensor when heads are stored apart."""
    if t.stride(-1) != 1:
        raise ValueError("the last KV dimension must be contiguous")
    if t.ndim == 3:
        return t, 0, 0
    if t.ndim != 4:
        raise ValueError(f"unsupported paged KV tensor rank {t.ndim}")
    nb, bs, h, d = t.shape
    if h == 1 or t.stride(2) == d:
        rows = t.reshape(nb, bs, h * d)
        if rows.data_ptr() != t.data_ptr() or rows.stride(2) != 1:
            raise ValueError("paged KV rows must be addressable in place")
        return rows, 0, 0
    return t, d, t.stride(2)


class PagedKVLayout:
    """Description of a registered paged KV cache (all layers).

    Builds the per-layer plane views, the chunk shape of each format, and (on
    CUDA) the native ``PagedLayout`` / ``ChunkLayout`` descriptors.
    """

    def __init__(self, kvcaches: KVCaches, use_mla: bool = False,
                 dsa_two_groups: bool = False,
                 fmt: Optional[KVCacheFormat] = None):
        self.fmt = fmt or KVCacheFormat.detect(kvcaches, use_mla, dsa_two_groups)
        if self.fmt == KVCacheFormat.UNDEFINED:
            raise ValueError("cannot detect the KV cache format")
        planes = self._split(kvcaches)
        self.planes: List[Plane] = planes
        first = planes[0].views[0]
        self.num_layers = len(planes[0].views)
        self.num_blocks = first.shape[0]
        self.block_size = first.shape[1]
        self.dtype = first.dtype
        self.device = first.device
        self.elem_size = first.element_size()
        for p in planes:
            for v in p.views:
                if v.shape[0] != self.num_blocks or v.shape[1] != self.block_size:
                    raise ValueError("all planes must share [num_blocks, block_size]")
                if v.dtype != self.dtype:
                    raise ValueError("mixed dtypes inside one KV layer group")
        self.num_slots = self.num_blocks * self.block_size
        self._native = None
        self._chunk_native = None
        self._slot_cache = {}

    # ------------------------------------------------------------------ split
    def _split(self, kvcaches: KVCaches) -> List[Plane]:
        fmt = self.fmt
        per_layer: List[List[torch.Tensor]] = []
        if fmt == KVCacheFormat.MERGED_KV:
            for t in kvcaches:
                if t.shape[0] == 2:
                    per_layer.append([t[0], t[1]])
                else:
                    per_layer.append([t[:, 0], t[:, 1]])
        elif fmt == KVCacheFormat.SEPARATE_KV and isinstance(kvcaches[0], torch.Tensor):
            k_all, v_all = kvcaches  # SGLang layer-concatenated
            per_layer = [[k_all[i], v_all[i]] for i in range(k_all.shape[0])]
        elif fmt == KVCacheFormat.MLA_FLAT:
            per_layer = [[t] for t in kvcaches]
        else:
            per_layer = [list(t) for t in kvcaches]
        nplanes = len(per_layer[0])
        planes = []
        for p in range(nplanes):
            got = [_as_rows(layer[p]) for layer in per_layer]
            views = [g[0] for g in got]
            v0 = views[0]
            row = v0.shape[2] * (v0.shape[3] if v0.ndim == 4 else 1)
            planes.append(Plane(views, row, v0.element_size(), got[0][1], got[0][2]))
        return planes

    # ----------------------------------------------------------- chunk format
    @property
    def num_planes(self) -> int:
        return len(self.planes)

    @property
    def row_bytes(self) -> List[int]:
        return [p.row_bytes for p in self.planes]

    @property
    def token_bytes(self) -> int:
        """Bytes of one token across all planes of one layer."""
        return sum(self.row_bytes)

    def chunk_shape(self, num_tokens: int) -> Tuple[int, ...]:
        """Shape of the chunk object holding ``num_tokens`` tokens."""
        if self.fmt.uses_2ltd_chunks:
            return (2, self.num_layers, num_tokens, self.planes[0].row_elems)
        return (1, self.num_layers, num_tokens, sum(p.row_elems for p in self.planes))

    def chunk_bytes(self, num_tokens: int) -> int:
        n = 1
        for s in self.chunk_shape(num_tokens):
            n *= s
        return n * self.elem_size

    def chunk_layout_params(self):
        """(plane_stride_t, layer_stride_t, token_stride, col_off) in bytes."""
        rb = self.row_bytes
        L = self.num_layers
        if self.fmt.uses_2ltd_chunks:
            return [L * rb[0]] * 2, rb[0], [rb[0]] * 2, [0, 0]
        row = sum(rb)
        offs, o = [], 0
        for r in rb:
            offs.append(o)
            o += r
        return [0] * len(rb), row, [row] * len(rb), offs

    # ------------------------------------------------------------- native side
    def native(self):
        """Native ``PagedLayout`` (device pointer table), built lazily."""
        if self._native is None:
            from .. import ops

            mod = ops.native()
            ptrs = []
            aligned = True
            for layer in range(self.num_layers):
                for p in self.planes:
                    v = p.views[layer]
                    ptrs.append(v.data_ptr())
                    aligned = aligned and (v.data_ptr() % 16 == 0)
            table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
            es = self.elem_size
            block_stride = [p.views[0].stride(0) * es for p in self.planes]
            slot_stride = [p.views[0].stride(1) * es for p in self.planes]
            seg_bytes = [p.seg_elems * es if p.segmented else 0 for p in self.planes]
            seg_stride = [p.seg_stride * es if p.segmented else 0 for p in self.planes]
            self._native = mod.PagedLayout(table, block_stride, slot_stride,
                                           self.row_bytes, self.block_size, self.num_slots,
                                           seg_bytes, seg_stride)
            self._native.set_bases_aligned(aligned)
        return self._native

    def chunk_native(self):
        if self._chunk_native is None:
            from .. import ops

            ps, ls, ts, co = self.chunk_layout_params()
            self._chunk_native = ops.native().ChunkLayout(ps, ls, ts, co)
        return self._chunk_native

    # ---------------------------------------------------------- torch oracle
    def _row_view(self, chunk: torch.Tensor, layer: int, p: int) -> torch.Tensor:
        """[T, E] view of plane p / layer of a chunk tensor."""
        if self.fmt.uses_2ltd_chunks:
            return chunk[p, layer]
        start = sum(q.row_elems for q in self.planes[:p])
        return chunk[0, layer, :, start:start + self.planes[p].row_elems]

    def gather_ref(self, chunk: torch.Tensor, slots: torch.Tensor,
                   layer_begin: int = 0, num_layers: Optional[int] = None,
                   chunk_layer_begin: int = 0, tok_off: int = 0) -> None:
        """PyTorch oracle: paged -> chunk for tokens with slot >= 0."""
        num_layers = self.num_layers - layer_begin if num_layers is None else num_layers
        slots = slots.to(self.device, torch.int64)
        valid = slots >= 0
        idx = torch.nonzero(valid).flatten()
        s = slots[idx]
        blk, off = s // self.block_size, s % self.block_size
        for li in range(num_layers):
            for p, plane in enumerate(self.planes):
                src = plane.rows(layer_begin + li, blk, off)
                dst = self._row_view(chunk, chunk_layer_begin + li, p)
                dst[idx.to(dst.device) + tok_off] = src.to(dst.device, dst.dtype)

    def scatter_ref(self, chunk: torch.Tensor, slots: torch.Tensor,
                    layer_begin: int = 0, num_layers: Optional[int] = None,
                    chunk_layer_begin: int = 0, tok_off: int = 0) -> None:
        """PyTorch oracle: chunk -> paged for tokens with slot >= 0."""
        num_layers = self.num_layers - layer_begin if num_layers is None else num_layers
        slots = slots.to(self.device, torch.int64)
        idx = torch.nonzero(slots >= 0).flatten()
        s = slots[idx]
        blk, off = s // self.block_size, s % self.block_size
        for li in range(num_layers):
            for p, plane in enumerate(self.planes):
                src = self._row_view(chunk, chunk_layer_begin + li, p)
                rows = src[idx.to(src.device) + tok_off].to(self.device, self.dtype)
                plane.set_rows(layer_begin + li, blk, off, rows)
