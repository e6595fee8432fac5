"""RoPE utilities for CacheBlend: fused K re-rotation with a start-up
self-check (reference lmcache_ascend/v1/blend/positional_encoding.py:95-250).

``FusedRope(old, new, k)`` rotates cached keys from the positions they were
stored at to the positions they take in the new prompt, in place, with the
native K8 kernel on CUDA tensors (oracle on CPU).  ``get_fused_rope``
validates the RoPE parameters (full rotary dim, no scaling) and checks the
fused op against plain RoPE before handing it out; it returns None when the
check fails so blending is disabled rather than silently wrong.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Optional

import torch

from ...ops import api
from ...ops.reference import make_cos_sin_cache, rope_apply_ref, rope_delta_ref
from ...utils.logging import init_logger

logger = init_logger(__name__)


class BasicRope:
    """Plain RoPE at given positions (fp32 math), for checks and reference."""

    def __init__(self, cos_sin_cache: torch.Tensor, head_size: int, is_neox: bool = True):
        self.cos_sin_cache = cos_sin_cache
        self.head_size = head_size
        self.is_neox = is_neox

    def __call__(self, positions, q, k):
        return (rope_apply_ref(positions.cpu(), q.cpu(), self.head_size, self.cos_sin_cache.cpu(),
                               self.is_neox).to(q.device, q.dtype),
                rope_apply_ref(positions.cpu(), k.cpu(), self.head_size, self.cos_sin_cache.cpu(),
                               self.is_neox).to(k.device, k.dtype))


class BasicReverseRope(BasicRope):
    """Undo RoPE: rotate from ``positions`` back to position 0."""

    def __call__(self, positions, q, k):
        zero = torch.zeros_like(positions)
        f = lambda x: rope_delta_ref(positions.cpu(), zero.cpu(), x.cpu(), self.head_size,
                                     self.cos_sin_cache.cpu(), self.is_neox).to(x.device, x.dtype)
        return f(q), f(k)


class FusedRope:
    """In-place K re-rotation old -> new positions (one kernel, one rounding)."""

    def __init__(self, cos_sin_cache: torch.Tensor, head_size: int, is_neox_style: bool = True):
        self.cos_sin_cache = cos_sin_cache
        self.head_size = head_size
        self.is_neox_style = is_neox_style

    def fused_encode(self, old_positions, new_positions, k):
        cache = self.cos_sin_cache
        if cache.device != k.device:
            cache = cache.to(k.device)
        api.rotary_embedding_k_fused(old_positions.to(k.device), new_positions.to(k.device), k,
                                     self.head_size, cache, self.is_neox_style)
        return k

    def __call__(self, old_positions, new_positions, k):
        return self.fused_encode(old_positions, new_positions, k)


def validate_rope_params(head_size: int, rotary_dim: int, max_position: int, base: float,
                         is_neox_style: bool = True, rope_scaling: Optional[Dict[str, Any]] = None,
                         dtype=None, partial_rotary_factor: float = 1.0) -> bool:
    if rotary_dim != head_size:
        logger.error("KV blending supports rotary_dim == head_size only")
        return False
    if rope_scaling is not None:
        logger.error("KV blending does not support rope scaling")
        return False
    if partial_rotary_factor != 1.0:
        logger.error("KV blending does not support a partial rotary factor")
        return False
    return True


def validate_reverse_correctness(rope: BasicRope, reverse_rope: BasicReverseRope,
                                 fused_rope: FusedRope, head_size: int, device) -> bool:
    hidden = head_size * 8
    n = 10
    g = torch.Generator().manual_seed(0)
    q = torch.rand(n, hidden, generator=g).to(device=device, dtype=torch.bfloat16)
    k = torch.rand(n, hidden, generator=g).to(device=device, dtype=torch.bfloat16)
    pos = torch.arange(n, device=device)
    q1, k1 = rope(pos, q.clone(), k.clone())
    q1, k1 = reverse_rope(pos, q1, k1)
    err_q = (q - q1).abs().max().item()
    err_k = (k - k1).abs().max().item()
    pos2 = torch.arange(100, 100 + n, device=device)
    _, k_at2 = rope(pos2, q.clone(), k.clone())
    _, k_at1 = rope(pos, q.clone(), k.clone())
    k_fused = fused_rope(pos, pos2, k_at1.clone())
    err_f = (k_at2.float() - k_fused.float()).abs().max().item()
    logger.info("rope self-check: reverse q %.4g k %.4g fused %.4g", err_q, err_k, err_f)
    return err_q < 0.1 and err_k < 0.1 and err_f < 0.1


def get_fused_rope(head_size: int, rotary_dim: int, max_position: int, base: float,
                   is_neox_style: bool = True, rope_scaling: Optional[Dict[str, Any]] = None,
                   dtype=None, partial_rotary_factor: float = 1.0,
                   device=None) -> Optional[Callable[..., Any]]:
    if not validate_rope_params(head_size, rotary_dim, max_position, base, is_neox_style,
                                rope_scaling, dtype, partial_rotary_factor):
        logger.warning("unsupported rope parameters: CacheBlend disabled")
        return None
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    cache = make_cos_sin_cache(max_position, rotary_dim, base).to(device)
    rope = BasicRope(cache, head_size, is_neox_style)
    fused = FusedRope(cache, head_size, is_neox_style)
    if not validate_reverse_correctness(rope, BasicReverseRope(cache, head_size, is_neox_style),
                                        fused, head_size, device):
        logger.error("fused/reverse rotary encoding failed its self-check: blending disabled")
        return None
    return fused
