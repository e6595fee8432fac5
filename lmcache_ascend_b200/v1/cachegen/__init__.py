"""CacheGen compression: per-layer quantisation + aligned prefix-code
entropy coding of KV chunks (serde for the remote tier).

Pipeline (the structure of upstream LMCache's CacheGen serde that the
reference drives, docs/cachegen/Cachegen.md:1-50, test usage in
tests/v1/test_cachegen_kernels.py):
  KV_2LTD chunk [2, L, T, C] -> per layer quantise to ``bins`` levels with a
  per-(layer, token) scale -> symbols [2L, T, C] uint8 -> per-(layer,
  channel) CDF -> encode -> bytes; decode reverses it.  ``bins`` is chosen
  per layer by ``QuantizationSpec`` ranges (more bins for early layers).
The entropy coder is the native K7 kernels on CUDA tensors and the
bit-identical oracle on CPU tensors.
"""

from __future__ import annotations

import struct
import warnings
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch

from ...ops import api, native

MAGIC = b"LMCG"
VERSION = 1
_DT = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}
_DT_ID = {v: k for k, v in _DT.items()}
_HDR = "<4sHIIIBH"    # magic, version, layers, tokens, channels, dtype id, groups
_GHDR = "<HII"        # per group: bins, rows, stream bytes
_LAZY_FIELDS = ("scales", "k_bins", "v_bins", "groups")


@dataclass
class QuantizationSpec:
    start_layer: int
    end_layer: int
    bins: int


@dataclass
class CacheGenConfig:
    nlayers: int
    kspecs: List[QuantizationSpec]
    vspecs: List[QuantizationSpec]

    @staticmethod
    def from_ranges(nlayers: int, k_ranges, v_ranges) -> "CacheGenConfig":
        return CacheGenConfig(nlayers, [QuantizationSpec(*r) for r in k_ranges],
                              [QuantizationSpec(*r) for r in v_ranges])

    @staticmethod
    def default(nlayers: int, early_bins: int = 32, late_bins: int = 16) -> "CacheGenConfig":
        """``early_bins`` levels for the first third of the layers, ``late_bins`` after
        (upstream LMCache uses 32 / 16)."""
        cut = max(1, nlayers // 3)
        return CacheGenConfig(nlayers, [QuantizationSpec(0, cut, early_bins),
                                        QuantizationSpec(cut, nlayers, late_bins)],
                              [QuantizationSpec(0, cut, early_bins),
                               QuantizationSpec(cut, nlayers, late_bins)])

    def bins(self, which: str, device=None) -> torch.Tensor:
        specs = self.kspecs if which == "k" else self.vspecs
        b = torch.zeros(self.nlayers, dtype=torch.int32)
        for s in specs:
            b[s.start_layer:min(s.end_layer, self.nlayers)] = s.bins
        if bool((b == 0).any()):
            raise ValueError(f"{which} quantisation specs do not cover every layer")
        return b.to(device) if device is not None else b


def quantize(x: torch.Tensor, bins: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x [L, T, C] float -> (symbols uint8 [L, T, C], scale fp32 [L, T]).
    Symmetric: level = round(x / scale) + half, half = bins // 2 - 1
    (fused native kernel on CUDA tensors, the same PyTorch expression on CPU)."""
    return api.cachegen_quantize(x, bins.to(torch.int32))


def dequantize(sym: torch.Tensor, scale: torch.Tensor, bins: torch.Tensor,
               dtype: torch.dtype) -> torch.Tensor:
    return api.cachegen_dequantize(sym, scale, bins.to(torch.int32), dtype)


def _group_order(row_bins: List[int]) -> Tuple[List[Tuple[int, List[int]]], List[int]]:
    """Rows grouped by bin count (ascending) and, per source row, its position
    in the grouped order."""
    groups = [(b, [r for r, x in enumerate(row_bins) if x == b]) for b in sorted(set(row_bins))]
    pos = [0] * len(row_bins)
    i = 0
    for _, rows in groups:
        for r in rows:
            pos[r] = i
            i += 1
    return groups, pos


def cdf_from_lengths(lengths: torch.Tensor) -> torch.Tensor:
    """Aligned CDF from code lengths [..., bins] (uint8, 0..12):
    start_s = sum_{r<s} 2^(16 - len_r); entry = start | len; last entry 0."""
    w = torch.pow(2, 16 - lengths.long())
    starts = torch.cumsum(w, dim=-1) - w
    ent = (starts & 0xFFF0) | lengths.long()
    last = torch.zeros(ent.shape[:-1] + (1,), dtype=torch.long, device=ent.device)
    out = torch.cat([ent, last], dim=-1)
    return torch.where(out >= 32768, out - 65536, out).to(torch.int16)


def _pack_nibbles(x: torch.Tensor) -> bytes:
    a = x.to(torch.uint8).flatten().cpu()
    if a.numel() % 2:
        a = torch.cat([a, torch.zeros(1, dtype=torch.uint8)])
    return ((a[0::2] << 4) | a[1::2]).numpy().tobytes()


def _unpack_nibbles(b: bytes, n: int) -> torch.Tensor:
    a = torch.frombuffer(bytearray(b), dtype=torch.uint8)
    out = torch.stack([a >> 4, a & 15], dim=1).flatten()
    return out[:n]


@dataclass
class CacheGenGroup:
    """Rows (of the 2L K-then-V layer rows) that share one bin count."""

    rows: List[int]
    bins: int
    code_lengths: torch.Tensor  # uint8 [n, C, bins]
    lengths: torch.Tensor       # int32 [n, C] bytes per stream
    streams: bytes


@dataclass
class CacheGenEncoded:
    num_layers: int
    num_tokens: int
    channels: int
    dtype: torch.dtype
    scales: torch.Tensor     # fp32 [2L, T]
    k_bins: torch.Tensor     # int32 [L]
    v_bins: torch.Tensor     # int32 [L]
    groups: List[CacheGenGroup]

    @classmethod
    def from_wire(cls, wire: bytes) -> "CacheGenEncoded":
        """Wrap a serialised payload.  ``to_bytes`` returns it unchanged and
        the sections (scales, bins, groups) are parsed on first access, so a
        payload that only travels (encode -> store, fetch -> decode) is never
        unpacked on the host."""
        L, T, C, dt = cls.peek_shape(wire)
        obj = cls.__new__(cls)
        obj.__dict__.update(num_layers=L, num_tokens=T, channels=C, dtype=dt, _wire=wire)
        return obj

    def __getattr__(self, name):
        wire = self.__dict__.get("_wire")
        if wire is not None and name in _LAZY_FIELDS:
            full = CacheGenEncoded.from_bytes(wire)
            for f in _LAZY_FIELDS:
                self.__dict__[f] = getattr(full, f)
            return self.__dict__[name]
        raise AttributeError(name)

    def to_bytes(self) -> bytes:
        wire = self.__dict__.get("_wire")
        if wire is not None:
            return wire
        L, T, C = self.num_layers, self.num_tokens, self.channels
        parts = [struct.pack(_HDR, MAGIC, VERSION, L, T, C, _DT_ID[self.dtype],
                             len(self.groups))]
        for t in (self.k_bins, self.v_bins, self.scales):
            parts.append(t.detach().cpu().contiguous().numpy().tobytes())
        for g in self.groups:
            cl = _pack_nibbles(g.code_lengths)
            parts.append(struct.pack(_GHDR, g.bins, len(g.rows), len(g.streams)))
            parts.append(torch.tensor(g.rows, dtype=torch.int32).numpy().tobytes())
            parts.append(g.lengths.detach().cpu().contiguous().numpy().tobytes())
            parts.append(cl)
            parts.append(g.streams)
        return b"".join(parts)

    @staticmethod
    def peek_shape(b: bytes) -> Tuple[int, int, int, torch.dtype]:
        """(layers, tokens, channels, dtype) from a payload's header."""
        magic, ver, L, T, C, dt, _ = struct.unpack(_HDR, b[:struct.calcsize(_HDR)])
        if magic != MAGIC or ver != VERSION:
            raise ValueError("not a CacheGen payload")
        return L, T, C, _DT[dt]

    @staticmethod
    def from_bytes(b: bytes) -> "CacheGenEncoded":
        n = struct.calcsize(_HDR)
        magic, ver, L, T, C, dt, ng = struct.unpack(_HDR, b[:n])
        if magic != MAGIC or ver != VERSION:
            raise ValueError("not a CacheGen payload")
        off = n

        def take(count, dtype, shape):
            nonlocal off
            a = np.frombuffer(b, dtype=dtype, count=count, offset=off).reshape(shape)
            off += count * np.dtype(dtype).itemsize
            return torch.from_numpy(a.copy())

        kb = take(L, np.int32, (L,))
        vb = take(L, np.int32, (L,))
        scales = take(2 * L * T, np.float32, (2 * L, T))
        groups = []
        for _ in range(ng):
            bins, nrows, slen = struct.unpack(_GHDR, b[off:off + 10])
            off += 10
            rows = take(nrows, np.int32, (nrows,)).tolist()
            lens = take(nrows * C, np.int32, (nrows, C))
            ncl = nrows * C * bins
            nb = (ncl + 1) // 2
            cl = _unpack_nibbles(b[off:off + nb], ncl).view(nrows, C, bins)
            off += nb
            groups.append(CacheGenGroup(rows, bins, cl, lens, b[off:off + slen]))
            off += slen
        return CacheGenEncoded(L, T, C, _DT[dt], scales, kb, vb, groups)


def _pack_nibbles_dev(x: torch.Tensor) -> torch.Tensor:
    """Device version of the code-length packing: two 4-bit lengths per byte,
    first in the high nibble (same bytes as ``_pack_nibbles``)."""
    a = x.to(torch.uint8).flatten()
    if a.numel() % 2:
        a = torch.cat([a, torch.zeros(1, dtype=torch.uint8, device=a.device)])
    return (a[0::2] << 4) | a[1::2]


def encode_kv(kv: torch.Tensor, config: CacheGenConfig) -> CacheGenEncoded:
    """kv: KV_2LTD chunk [2, L, T, C] (device or host).  One quantise launch
    writes the symbols of rows sharing a bin count next to each other, so
    every group's CDF and encode run on a contiguous slice.  On the device
    the streams are then packed back to back by one compaction kernel and
    the whole payload (scales, lengths, code lengths, streams) leaves the GPU
    in one copy, after one small read of the per-group stream totals."""
    _, L, T, C = kv.shape
    dev = kv.device
    kb, vb = config.bins("k"), config.bins("v")
    row_bins_t = torch.cat([kb, vb]).to(torch.int32)
    row_bins = row_bins_t.tolist()
    order, pos = _group_order(row_bins)
    sym, scale = api.cachegen_quantize(kv.reshape(2 * L, T, C), row_bins_t.to(dev),
                                       torch.tensor(pos, dtype=torch.int32, device=dev))
    cap = ((T * 12 + 7) // 8 + 4) // 4 * 4
    enc_out = []  # per group: (bins, rows, stream slots, lengths, code lengths)
    off = 0
    for bins, rows in order:
        sg = sym[off:off + len(rows)]
        off += len(rows)
        cdf = api.calculate_cdf(sg, bins)
        out = torch.empty(len(rows), C, cap, dtype=torch.uint8, device=dev)
        lens = torch.empty(len(rows), C, dtype=torch.int32, device=dev)
        api.encode_fast_new(cdf, sg, out, lens)
        code_len = (cdf[..., :bins].to(torch.int32) & 0xF).to(torch.uint8)
        enc_out.append((bins, rows, out, lens, code_len))
    if dev.type != "cuda":
        groups = []
        for bins, rows, out, lens, code_len in enc_out:
            mask = torch.arange(cap).unsqueeze(0) < lens.view(-1, 1)
            groups.append(CacheGenGroup(rows, bins, code_len, lens,
                                        out.view(-1, cap)[mask].numpy().tobytes()))
        return CacheGenEncoded(L, T, C, kv.dtype, scale.float(), kb, vb, groups)
    from ...ops import native

    all_lens = torch.cat([g[3].view(-1) for g in enc_out])
    ends = torch.cumsum(all_lens.to(torch.int64), 0)
    offsets = ends - all_lens
    counts = [g[3].numel() for g in enc_out]
    bounds = torch.tensor(counts, dtype=torch.int64).cumsum(0) - 1
    totals = ends[bounds.to(dev)].cpu().tolist()  # the one device read before the copy
    group_bytes = [t - (totals[i - 1] if i else 0) for i, t in enumerate(totals)]
    streams = torch.empty(max(1, totals[-1]), dtype=torch.uint8, device=dev)
    first = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)[:-1].tolist()),
                         dtype=torch.int64, device=dev)
    native().cachegen_compact(
        torch.tensor([g[2].data_ptr() for g in enc_out], dtype=torch.int64, device=dev),
        torch.full((len(enc_out),), cap, dtype=torch.int64, device=dev), first, all_lens,
        offsets, streams)
    # The payload is laid out on the device in its wire order (the layout
    # ``to_bytes`` writes): the host-known headers go over in one small copy,
    # the device sections are concatenated around them, one copy brings the
    # whole payload back.
    head = [struct.pack(_HDR, MAGIC, VERSION, L, T, C, _DT_ID[kv.dtype], len(enc_out)),
            kb.to(torch.int32).numpy().tobytes(), vb.to(torch.int32).numpy().tobytes()]
    ghead = [struct.pack(_GHDR, bins, len(rows), nb) + np.asarray(rows, np.int32).tobytes()
             for (bins, rows, _, _, _), nb in zip(enc_out, group_bytes)]
    known = b"".join(head + ghead)
    known_d = torch.frombuffer(bytearray(known), dtype=torch.uint8).to(dev)
    h0 = sum(len(h) for h in head)
    pieces = [known_d[:h0], scale.float().contiguous().view(torch.uint8).view(-1)]
    ho, so = h0, 0
    for (bins, rows, _, lens, code_len), gh, nb in zip(enc_out, ghead, group_bytes):
        pieces += [known_d[ho:ho + len(gh)], lens.contiguous().view(torch.uint8).view(-1),
                   _pack_nibbles_dev(code_len), streams[so:so + nb]]
        ho += len(gh)
        so += nb
    wire_d = torch.cat(pieces)
    host = torch.empty(wire_d.numel(), dtype=torch.uint8, pin_memory=True)
    host.copy_(wire_d, non_blocking=True)
    torch.cuda.current_stream(dev).synchronize()
    return CacheGenEncoded.from_wire(host.numpy().tobytes())


def decode_kv_bytes(data: bytes, device="cpu", out: Optional[torch.Tensor] = None
                    ) -> torch.Tensor:
    """Decode a serialised payload (``CacheGenEncoded.to_bytes``) straight
    from bytes: on the device the payload goes over in one copy and every
    section is used in place (no per-group transfers)."""
    dev = torch.device(device)
    if dev.type != "cuda":
        return decode_kv(CacheGenEncoded.from_bytes(data), dev, out)
    n = struct.calcsize(_HDR)
    magic, ver, L, T, C, dt, ng = struct.unpack(_HDR, data[:n])
    if magic != MAGIC or ver != VERSION:
        raise ValueError("not a CacheGen payload")
    dtype = _DT[dt]
    kb = torch.from_numpy(np.frombuffer(data, np.int32, count=L, offset=n).copy())
    vb = torch.from_numpy(np.frombuffer(data, np.int32, count=L, offset=n + 4 * L).copy())
    # one copy straight from the payload's memory (the driver stages a
    # pageable source through its own pinned buffers, pipelined with the DMA:
    # measured faster than a host copy into pinned memory followed by a DMA)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # read-only source buffer: nothing writes it
        payload = torch.frombuffer(data, dtype=torch.uint8).to(dev)
    off = n + 8 * L
    scales = payload[off:off + 8 * L * T].clone().view(torch.float32).view(2 * L, T)
    off += 8 * L * T
    sym = torch.empty(2 * L, T, C, dtype=torch.uint8, device=dev)
    pos = [0] * (2 * L)
    row0 = 0
    for _ in range(ng):
        bins, nrows, slen = struct.unpack(_GHDR, data[off:off + 10])
        off += 10
        rows = np.frombuffer(data, dtype=np.int32, count=nrows, offset=off).tolist()
        off += 4 * nrows
        lens = payload[off:off + 4 * nrows * C].clone().view(torch.int32)
        off += 4 * nrows * C
        ncl = nrows * C * bins
        packed = payload[off:off + (ncl + 1) // 2]
        off += (ncl + 1) // 2
        cdf = native().cachegen_cdf_from_lengths(packed, nrows, C, bins)  # one launch
        stream = payload[off:off + slen] if slen else torch.zeros(1, dtype=torch.uint8,
                                                                  device=dev)
        off += slen
        cum = torch.cumsum(lens, 0).to(torch.int32).view(nrows, C)
        api.decode_fast_prefsum(cdf, stream, cum, sym[row0:row0 + nrows])
        for i, r in enumerate(rows):
            pos[r] = row0 + i
        row0 += nrows
    # small host tables go over from pinned memory without a synchronisation
    row_bins = torch.cat([kb, vb]).to(torch.int32).pin_memory().to(dev, non_blocking=True)
    src = torch.tensor(pos, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
    direct = out is not None and out.is_contiguous() and out.dtype == dtype and \
        out.device == dev
    y = api.cachegen_dequantize(sym, scales, row_bins, dtype, row_src=src,
                                out=out.view(2 * L, T, C) if direct else None)
    res = y.view(2, L, T, C)
    if out is not None and not direct:
        out.copy_(res)
        return out
    return out if direct else res


def decode_kv(enc: CacheGenEncoded, device="cpu", out: Optional[torch.Tensor] = None
              ) -> torch.Tensor:
    """Decode every group into its slice of the grouped symbol buffer, then one
    dequantise launch writes the [2, L, T, C] chunk (into ``out`` when given)."""
    dev = torch.device(device)
    if dev.type == "cuda" and enc.__dict__.get("_wire") is not None \
            and "groups" not in enc.__dict__:
        return decode_kv_bytes(enc.__dict__["_wire"], dev, out)
    L, T, C = enc.num_layers, enc.num_tokens, enc.channels
    sym = torch.empty(2 * L, T, C, dtype=torch.uint8, device=dev)
    pos = [0] * (2 * L)
    off = 0
    for g in enc.groups:
        cdf = cdf_from_lengths(g.code_lengths.to(dev))
        stream = torch.frombuffer(bytearray(g.streams), dtype=torch.uint8).to(dev) \
            if g.streams else torch.zeros(1, dtype=torch.uint8, device=dev)
        cum = g.lengths.view(-1).cumsum(0).to(torch.int32).view(len(g.rows), C).to(dev)
        api.decode_fast_prefsum(cdf, stream, cum, sym[off:off + len(g.rows)])
        for i, r in enumerate(g.rows):
            pos[r] = off + i
        off += len(g.rows)
    row_bins = torch.cat([enc.k_bins, enc.v_bins]).to(torch.int32)
    src = torch.tensor(pos, dtype=torch.int32, device=dev)
    direct = out is not None and out.is_contiguous() and out.dtype == enc.dtype and \
        out.device == dev and out.dtype in (torch.float16, torch.bfloat16, torch.float32)
    y = api.cachegen_dequantize(sym, enc.scales.to(dev), row_bins, enc.dtype, row_src=src,
                                out=out.view(2 * L, T, C) if direct else None)
    res = y.view(2, L, T, C)
    if out is not None and not direct:
        out.copy_(res)
        return out
    return out if direct else res
