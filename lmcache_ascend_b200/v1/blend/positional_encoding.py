"""RoPE utilities for CacheBlend: fused K re-rotation with a start-up
self-check (reference lmcache_ascend/v1/blend/positional_encoding.py:95-250).

``FusedRope(old, new, k)`` rotates cached keys from the positions they were
stored at to the positions they take in the new prompt, in place, with the
native K8 kernel on CUDA tensors (oracle on CPU).  ``get_fused_rope``
refuses RoPE variants the kernel does not implement (partial rotary dim,
scaling) and checks the fused op on random keys and positions against the
oracle before handing it out; it returns None when the check fails so
blending is disabled rather than silently wrong.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, List, Optional, Tuple

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


def unsupported_rope(head_size: int, rotary_dim: int, rope_scaling: Optional[Dict[str, Any]],
                     partial_rotary_factor: float) -> List[str]:
    """Reasons the fused re-rotation cannot serve this model's RoPE (empty
    list: supported).  The kernel rotates the whole head with unscaled
    frequencies, so a partial rotary dim or any rope scaling rules it out."""
    why = []
    if rotary_dim != head_size or partial_rotary_factor != 1.0:
        why.append(f"partial rotary embedding (rotary_dim {rotary_dim} of {head_size}, "
                   f"factor {partial_rotary_factor})")
    if rope_scaling:
        why.append(f"rope scaling {rope_scaling}")
    return why


def self_check(fused_rope: "FusedRope", max_position: int, device, heads: int = 4,
               tokens: int = 64, seed: int = 1234) -> Tuple[bool, float, float]:
    """Re-rotate random bf16 keys from random positions to random new ones
    and compare with keys rotated at the new positions directly (oracle),
    then rotate back and compare with the start.

    Tolerance: each side of the comparison went through at most two bf16
    roundings (2^-8 relative each) plus the fp32 angle error, which grows
    with the position (about position x 2^-23 radians), all relative to the
    largest key magnitude.  Returns (passed, max error, tolerance)."""
    D = fused_rope.head_size
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(tokens, heads * D, generator=g).to(torch.bfloat16)
    half = max(1, max_position // 2)
    old = torch.randint(0, half, (tokens,), generator=g)
    new = torch.randint(0, half, (tokens,), generator=g) + torch.randint(0, 2, (tokens,),
                                                                        generator=g) * (half - 1)
    new = new.clamp(max=max_position - 1)
    cache = fused_rope.cos_sin_cache.cpu()
    neox = fused_rope.is_neox_style
    at_old = rope_apply_ref(old, k.float(), D, cache, neox).to(torch.bfloat16)
    at_new = rope_apply_ref(new, k.float(), D, cache, neox).to(torch.bfloat16)
    moved = fused_rope(old.to(device), new.to(device), at_old.clone().to(device)).cpu()
    back = fused_rope(new.to(device), old.to(device), moved.clone().to(device)).cpu()
    scale = float(k.float().abs().max())
    tol = (2.0 ** -7 + max_position * 2.0 ** -23) * scale * 2
    err = max(float((moved.float() - at_new.float()).abs().max()),
              float((back.float() - at_old.float()).abs().max()))
    return err <= tol, err, tol


def get_fused_rope(head_size: int, rotary_dim: int, max_position: int, base: float,
                   is_neox_style: bool = True, rope_scaling: Optional[Dict[str, Any]] = None,
                   dtype=None, partial_rotary_factor: float = 1.0,
                   device=None) -> Optional[Callable[..., Any]]:
    """The fused K re-rotation for this RoPE, or None (blending disabled)
    when the RoPE is not supported or the op fails its self-check."""
    why = unsupported_rope(head_size, rotary_dim, rope_scaling, partial_rotary_factor)
    if why:
        logger.warning("CacheBlend disabled: %s", "; ".join(why))
        return None
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    cache = make_cos_sin_cache(max_position, rotary_dim, base).to(device)
    fused = FusedRope(cache, head_size, is_neox_style)
    ok, err, tol = self_check(fused, max_position, device)
    logger.info("fused RoPE self-check: max error %.3g (tolerance %.3g)", err, tol)
    if not ok:
        logger.error("fused RoPE failed its self-check (%.3g > %.3g): blending disabled",
                     err, tol)
        return None
    return fused
