"""PyTorch / NumPy oracles of the native kernels.

Used (a) as the numerics reference of the GPU tests and (b) as the CPU
implementation when tensors live on the host (CPU-only deployments and the
CPU test tier).  They implement the same formats as the CUDA kernels:

* CacheGen (``cachegen_kernels.cu``): aligned power-of-two CDF with the code
  length in the low 4 bits of each entry, MSB-first prefix codes, decode
  from an inclusive prefix sum of stream lengths;
* RoPE delta re-rotation (``pos_kernels.cu``).
"""

from __future__ import annotations

from typing import List, Tuple

import numpy as np
import torch

MAX_BINS = 256


# ---------------------------------------------------------------------------
# CacheGen
# ---------------------------------------------------------------------------
def cdf_assign(counts: List[int]) -> List[int]:
    """Aligned CDF of one channel (exact mirror of ``cdf_assign`` in C++).

    Returns bins + 1 uint16 entries: ``(start & 0xFFF0) | code_len``; the
    last entry (0) stands for 0x10000.
    """
    bins = len(counts)
    if bins == 1:
        return [0, 0]
    total = sum(int(c) for c in counts)
    den = 2 * total + bins
    out = [0] * (bins + 1)
    pos = 0
    for s in range(bins):
        k = bins - s
        R = 65536 - pos
        if k == 1:
            w = R
        else:
            x = (2 * int(counts[s]) + 1) * 65536
            wd = 16
            while wd < 32768 and den * (2 * wd) <= x:
                wd <<= 1
            if wd < 32768 and 2 * x >= 3 * den * wd:
                wd <<= 1
            ed = wd.bit_length() - 1
            maxw = 32768 if pos == 0 else (pos & -pos)
            best_e, best_d = -1, 1 << 30
            e = 4
            while (1 << e) <= maxw:
                cand = 1 << e
                if cand >= R:
                    break
                rem = R - cand
                if bin(rem).count("1") <= k - 1 and (k - 1) <= rem // 16:
                    d = abs(e - ed)
                    if d < best_d or (d == best_d and e > best_e):
                        best_d, best_e = d, e
                e += 1
            w = (1 << best_e) if best_e >= 0 else 16
        length = 16 - (w.bit_length() - 1)
        out[s] = (pos & 0xFFF0) | length
        pos += w
    out[bins] = 0
    return out


def calculate_cdf_ref(symbols: torch.Tensor, n_bins: int) -> torch.Tensor:
    """symbols [L, T, C] uint8 -> int16 [L, C, n_bins + 1]."""
    s = symbols.detach().cpu().numpy().astype(np.int64)
    L, T, C = s.shape
    s = np.minimum(s, n_bins - 1)
    out = np.zeros((L, C, n_bins + 1), dtype=np.uint16)
    for l in range(L):
        for c in range(C):
            counts = np.bincount(s[l, :, c], minlength=n_bins)[:n_bins]
            out[l, c] = cdf_assign(counts.tolist())
    return torch.from_numpy(out.view(np.int16).copy())


def _code_tables(cdf_row: np.ndarray) -> Tuple[List[int], List[int]]:
    bins = len(cdf_row) - 1
    starts = [int(v) & 0xFFF0 for v in cdf_row[:bins]] + [65536]
    codes, lens = [], []
    for s in range(bins):
        w = starts[s + 1] - starts[s]
        if w <= 0:
            codes.append(0)
            lens.append(-1)
            continue
        e = w.bit_length() - 1
        ln = 16 - e
        lens.append(ln)
        codes.append(0 if ln == 0 else starts[s] >> (16 - ln))
    return codes, lens


def encode_ref(cdf: torch.Tensor, symbols: torch.Tensor, cap: int
               ) -> Tuple[torch.Tensor, torch.Tensor]:
    """-> (bytes [L, C, cap] uint8, lengths [L, C] int32)."""
    c = cdf.detach().cpu().numpy().view(np.uint16) if cdf.dtype == torch.int16 else \
        cdf.detach().cpu().numpy().astype(np.int64).astype(np.uint16)
    s = symbols.detach().cpu().numpy().astype(np.int64)
    L, T, C = s.shape
    bins = c.shape[2] - 1
    out = np.zeros((L, C, cap), dtype=np.uint8)
    lens = np.zeros((L, C), dtype=np.int32)
    for l in range(L):
        for ch in range(C):
            codes, cl = _code_tables(c[l, ch])
            acc, nb, buf = 0, 0, bytearray()
            for t in range(T):
                sym = min(int(s[l, t, ch]), bins - 1)
                ln = cl[sym]
                if ln < 0:
                    raise ValueError(f"symbol {sym} has zero width in the CDF")
                acc = (acc << ln) | codes[sym]
                nb += ln
                while nb >= 8:
                    buf.append((acc >> (nb - 8)) & 0xFF)
                    nb -= 8
                    acc &= (1 << nb) - 1
            if nb:
                buf.append((acc << (8 - nb)) & 0xFF)
            n = min(len(buf), cap)
            out[l, ch, :n] = np.frombuffer(bytes(buf[:n]), dtype=np.uint8)
            lens[l, ch] = n
    return torch.from_numpy(out), torch.from_numpy(lens)


def decode_ref(cdf: torch.Tensor, bytestream: torch.Tensor, cum_lengths: torch.Tensor,
               num_tokens: int) -> torch.Tensor:
    """Inverse of ``encode_ref`` with concatenated streams -> [L, T, C] uint8."""
    c = cdf.detach().cpu().numpy().view(np.uint16) if cdf.dtype == torch.int16 else \
        cdf.detach().cpu().numpy().astype(np.int64).astype(np.uint16)
    b = bytestream.detach().cpu().numpy().astype(np.uint8).tobytes()
    cl = cum_lengths.detach().cpu().numpy().astype(np.int64).reshape(-1)
    L, C, bp1 = c.shape
    bins = bp1 - 1
    out = np.zeros((L, num_tokens, C), dtype=np.uint8)
    for l in range(L):
        for ch in range(C):
            idx = l * C + ch
            b0 = 0 if idx == 0 else int(cl[idx - 1])
            stream = b[b0:int(cl[idx])]
            starts = [int(v) & 0xFFF0 for v in c[l, ch, :bins]]
            lens = [int(v) & 0xF for v in c[l, ch, :bins]]
            bits = int.from_bytes(stream, "big") if stream else 0
            nbits = 8 * len(stream)
            pos = 0
            for t in range(num_tokens):
                # next 16 bits (zero padded)
                if pos >= nbits:
                    v = 0
                else:
                    sh = nbits - pos - 16
                    v = (bits >> sh) & 0xFFFF if sh >= 0 else (bits << -sh) & 0xFFFF
                lo, hi = 0, bins - 1
                while lo < hi:
                    mid = (lo + hi + 1) >> 1
                    if starts[mid] <= v:
                        lo = mid
                    else:
                        hi = mid - 1
                out[l, t, ch] = lo
                pos += lens[lo]
    return torch.from_numpy(out)


# ---------------------------------------------------------------------------
# RoPE delta re-rotation
# ---------------------------------------------------------------------------
def rope_delta_ref(old_pos: torch.Tensor, new_pos: torch.Tensor, key: torch.Tensor,
                   head_size: int, cos_sin_cache: torch.Tensor, is_neox: bool
                   ) -> torch.Tensor:
    """fp32 reference: rotate K from ``old_pos`` to ``new_pos`` (returns a copy)."""
    T = key.shape[0]
    k = key.reshape(T, -1, head_size).float().clone()
    rot = cos_sin_cache.shape[1]
    half = rot // 2
    cs = cos_sin_cache.float()
    cn, sn = cs[new_pos.long(), :half], cs[new_pos.long(), half:]
    co, so = cs[old_pos.long(), :half], cs[old_pos.long(), half:]
    cd = (cn * co + sn * so)[:, None, :]
    sd = (sn * co - cn * so)[:, None, :]
    if is_neox:
        x1, x2 = k[..., :half].clone(), k[..., half:rot].clone()
        k[..., :half] = x1 * cd - x2 * sd
        k[..., half:rot] = x2 * cd + x1 * sd
    else:
        x1, x2 = k[..., 0:rot:2].clone(), k[..., 1:rot:2].clone()
        k[..., 0:rot:2] = x1 * cd - x2 * sd
        k[..., 1:rot:2] = x2 * cd + x1 * sd
    return k.reshape(key.shape)


def rope_apply_ref(pos: torch.Tensor, key: torch.Tensor, head_size: int,
                   cos_sin_cache: torch.Tensor, is_neox: bool) -> torch.Tensor:
    """Plain RoPE at ``pos`` (fp32): rotation from position 0."""
    zero = torch.zeros_like(pos)
    return rope_delta_ref(zero, pos, key, head_size, cos_sin_cache, is_neox)


def make_cos_sin_cache(max_pos: int, rot_dim: int, base: float = 10000.0,
                       dtype=torch.float32) -> torch.Tensor:
    """vLLM layout: [max_pos, rot_dim], first half cos, second half sin."""
    inv = 1.0 / (base ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).to(dtype)
