"""K7 CacheGen: exact bitstreams (reference test vectors of
tests/v1/test_cachegen_kernels.py in LMCache-Ascend), CDF construction,
encode->decode round trips; CPU oracle always, CUDA kernels on GPU."""

import pytest
import torch

from lmcache_ascend_b200 import ops
from lmcache_ascend_b200.ops import reference as R

CAP = 256
HAVE_GPU = torch.cuda.is_available()


def _expected_binary(bits):
    s = "".join(f"{t:0{bits}b}" for t in range(2 ** bits))
    if len(s) % 8:
        s += "0" * (8 - len(s) % 8)
    return [int(s[i:i + 8], 2) for i in range(0, len(s), 8)]


def _uniform_cdf(bits, layers, channels, with_len=False):
    bins = 2 ** bits + 1
    f = 0x10000 // (bins - 1)
    row = [(b * f) & 0xFFFF for b in range(bins)]
    if with_len:
        row = [v | bits for v in row]
    t = torch.tensor(row, dtype=torch.int32).to(torch.int16)
    return t.view(1, 1, bins).expand(layers, channels, bins).contiguous()


def _symbols(bits, layers, channels):
    n = 2 ** bits
    s = torch.arange(n, dtype=torch.uint8).view(1, n, 1).expand(layers, n, channels)
    return s.contiguous()


def _encode(cdf, sym, cap, device):
    if device == "cpu":
        return R.encode_ref(cdf, sym, cap)
    out = torch.zeros(sym.shape[0], sym.shape[2], cap, dtype=torch.uint8, device=device)
    lens = torch.zeros(sym.shape[0], sym.shape[2], dtype=torch.int32, device=device)
    ops.native().encode_fast_new(cdf.to(device), sym.to(device), out, lens)
    torch.cuda.synchronize()
    return out.cpu(), lens.cpu()


def _decode(cdf, stream, cum, T, device):
    if device == "cpu":
        return R.decode_ref(cdf, stream, cum, T)
    L, C = cdf.shape[0], cdf.shape[1]
    out = torch.zeros(L, T, C, dtype=torch.uint8, device=device)
    ops.native().decode_fast_prefsum(cdf.to(device), stream.to(device), cum.to(device), out)
    torch.cuda.synchronize()
    return out.cpu()


DEVICES = ["cpu"] + (["cuda"] if HAVE_GPU else [])
gpu_param = pytest.param("cuda", marks=pytest.mark.gpu)


def devices():
    return ["cpu", gpu_param]


@pytest.mark.parametrize("device", devices())
@pytest.mark.parametrize("layers", [1, 2])
@pytest.mark.parametrize("channels", [1, 32, 256])
@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6])
def test_basic_encode(device, layers, channels, bits):
    cdf = _uniform_cdf(bits, layers, channels)
    sym = _symbols(bits, layers, channels)
    out, lens = _encode(cdf, sym, CAP, device)
    exp = _expected_binary(bits)
    assert (lens == len(exp)).all()
    want = torch.zeros(CAP, dtype=torch.uint8)
    want[:len(exp)] = torch.tensor(exp, dtype=torch.uint8)
    assert (out == want).all()


@pytest.mark.parametrize("device", devices())
def test_basic_non_uniform_encode(device):
    cdf = torch.tensor([0x0000, 0x8000, 0x8000, 0xC000, 0x10000], dtype=torch.int32)
    cdf = (cdf & 0xFFFF).to(torch.int16).view(1, 1, 5)
    sym = torch.tensor([0, 0, 2, 3], dtype=torch.uint8).view(1, 4, 1)
    out, lens = _encode(cdf, sym, 4, device)
    assert int(out[0, 0, 0]) == int("00101100", 2)
    assert int(lens[0, 0]) == 1


@pytest.mark.parametrize("device", devices())
@pytest.mark.parametrize("layers", [1, 2])
@pytest.mark.parametrize("channels", [32, 256])
@pytest.mark.parametrize("bits", [2, 3, 4, 5])
def test_basic_decode(device, layers, channels, bits):
    stream = _expected_binary(bits)
    streams = torch.tensor(stream * layers * channels, dtype=torch.uint8)
    cum = torch.tensor([len(stream)] * layers * channels, dtype=torch.int32).cumsum(0)
    cum = cum.to(torch.int32).view(layers, channels)
    cdf = _uniform_cdf(bits, layers, channels, with_len=True)
    out = _decode(cdf, streams, cum, 2 ** bits, device)
    assert torch.equal(out, _symbols(bits, layers, channels))


def test_cdf_assign_properties():
    import random

    rnd = random.Random(0)
    for bins in [1, 2, 3, 5, 16, 17, 32, 33, 64, 200, 256]:
        for _ in range(20):
            counts = [rnd.choice([0, 0, 1, 5, 100, 10000]) for _ in range(bins)]
            cdf = R.cdf_assign(counts)
            starts = [v & 0xFFF0 for v in cdf[:bins]] + [65536]
            lens = [v & 0xF for v in cdf[:bins]]
            for s in range(bins):
                w = starts[s + 1] - starts[s]
                assert w > 0 and (w & (w - 1)) == 0, (bins, counts, cdf)
                assert starts[s] % w == 0  # aligned
                assert lens[s] == 16 - (w.bit_length() - 1)
                assert lens[s] <= 12


@pytest.mark.parametrize("device", devices())
@pytest.mark.parametrize("bins", [16, 32, 64, 256])
def test_cdf_then_round_trip(device, bins):
    g = torch.Generator().manual_seed(bins)
    L, T, C = 3, 200, 64
    # skewed symbols (quantised gaussian-like)
    x = torch.randn(L, T, C, generator=g) * (bins / 8) + bins / 2
    sym = x.clamp(0, bins - 1).round().to(torch.uint8)
    if device == "cpu":
        cdf = R.calculate_cdf_ref(sym, bins)
    else:
        cdf = ops.native().calculate_cdf(sym.cuda(), bins).cpu()
        assert torch.equal(cdf, R.calculate_cdf_ref(sym, bins))
    cap = T * 12 // 8 + 2
    out, lens = _encode(cdf, sym, cap, device)
    # compression: skewed data must beat the fixed-width code
    width = (bins - 1).bit_length()
    assert lens.sum().item() < L * C * T * width / 8
    streams = torch.cat([out[l, c, :lens[l, c]] for l in range(L) for c in range(C)])
    cum = lens.view(-1).cumsum(0).to(torch.int32).view(L, C)
    dec = _decode(cdf, streams, cum, T, device)
    assert torch.equal(dec, sym)


@pytest.mark.gpu
def test_gpu_encode_matches_cpu_bitstream():
    g = torch.Generator().manual_seed(7)
    L, T, C, bins = 2, 256, 96, 32
    sym = torch.randint(0, bins, (L, T, C), generator=g, dtype=torch.uint8)
    cdf = R.calculate_cdf_ref(sym, bins)
    cap = 400
    a, la = _encode(cdf, sym, cap, "cpu")
    b, lb = _encode(cdf, sym, cap, "cuda")
    assert torch.equal(la, lb) and torch.equal(a, b)


def _torch_quantize(x, bins):
    half = (bins // 2 - 1).view(-1, 1, 1).float()
    amax = x.float().abs().amax(dim=-1, keepdim=True).clamp_min(1e-8)
    sc = amax / half
    q = torch.minimum((torch.round(x.float() / sc) + half).clamp_min(0), 2 * half)
    return q.to(torch.uint8), sc.squeeze(-1)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("C", [1024, 100])
def test_gpu_quantize_dequantize_match_torch(dtype, C):
    from lmcache_ascend_b200.ops import api

    g = torch.Generator().manual_seed(C)
    R_, T = 6, 77
    x = (torch.randn(R_, T, C, generator=g) * torch.rand(1, 1, C, generator=g) * 2).to(dtype)
    bins = torch.tensor([32, 32, 16, 16, 256, 4], dtype=torch.int32)
    want_q, want_s = _torch_quantize(x, bins)
    perm = torch.tensor([3, 0, 5, 1, 4, 2], dtype=torch.int32)
    q, s = api.cachegen_quantize(x.cuda(), bins.cuda(), perm.cuda())
    assert torch.equal(s.cpu(), want_s)
    assert torch.equal(q.cpu()[perm.long()], want_q)
    y = api.cachegen_dequantize(q, s, bins.cuda(), dtype, row_src=perm.cuda())
    half = (bins // 2 - 1).view(-1, 1, 1).float()
    want_y = ((want_q.float() - half) * want_s.unsqueeze(-1)).to(dtype)
    assert torch.equal(y.cpu(), want_y)


@pytest.mark.gpu
@pytest.mark.parametrize("bins", [16, 32, 256])
def test_gpu_codec_odd_shapes_and_misaligned_streams(bins):
    # T not a multiple of the 64-token tile, C not a multiple of 16 or 128,
    # cap not a multiple of 4, stream buffer starting 1 byte past an allocation
    g = torch.Generator().manual_seed(bins + 1)
    L, T, C = 2, 203, 150
    x = torch.randn(L, T, C, generator=g) * (bins / 7) + bins / 2
    sym = x.clamp(0, bins - 1).round().to(torch.uint8)
    cdf = ops.native().calculate_cdf(sym.cuda(), bins).cpu()
    assert torch.equal(cdf, R.calculate_cdf_ref(sym, bins))
    cap = T * 12 // 8 + 3
    a, la = _encode(cdf, sym, cap, "cpu")
    b, lb = _encode(cdf, sym, cap, "cuda")
    assert torch.equal(la, lb) and torch.equal(a, b)
    streams = torch.cat([a[l, c, :la[l, c]] for l in range(L) for c in range(C)])
    cum = la.view(-1).cumsum(0).to(torch.int32).view(L, C)
    buf = torch.zeros(streams.numel() + 1, dtype=torch.uint8, device="cuda")
    buf[1:] = streams.cuda()
    out = torch.zeros(L, T, C, dtype=torch.uint8, device="cuda")
    ops.native().decode_fast_prefsum(cdf.cuda(), buf[1:], cum.cuda(), out)
    assert torch.equal(out.cpu(), sym)


@pytest.mark.gpu
def test_gpu_cachegen_kv_round_trip_matches_cpu():
    from lmcache_ascend_b200.v1.cachegen import CacheGenConfig, decode_kv, encode_kv

    g = torch.Generator().manual_seed(3)
    L, T, C = 6, 256, 256
    kv = (torch.randn(2, L, T, C, generator=g) *
          (0.5 + 1.5 * torch.rand(1, 1, 1, C, generator=g))).to(torch.bfloat16)
    cfg = CacheGenConfig.default(L)
    e_cpu = encode_kv(kv, cfg)
    e_gpu = encode_kv(kv.cuda(), cfg)
    assert e_cpu.to_bytes() == e_gpu.to_bytes()
    out = torch.empty(2, L, T, C, dtype=torch.bfloat16, device="cuda")
    y = decode_kv(e_gpu, device="cuda", out=out)
    assert y.data_ptr() == out.data_ptr()
    assert torch.equal(y.cpu(), decode_kv(e_cpu))


@pytest.mark.gpu
@pytest.mark.parametrize("bins", [1, 16, 33, 256])
def test_cdf_from_packed_lengths_kernel_matches_tensor_ops(bins):
    """The fused rebuild of CDF rows from the serialised 4-bit code lengths
    gives the same int16 rows as the tensor-op form (``cdf_from_lengths``)."""
    from lmcache_ascend_b200.ops import native
    from lmcache_ascend_b200.v1.cachegen import _pack_nibbles_dev, cdf_from_lengths

    g = torch.Generator().manual_seed(bins)
    rows, C = 3, 37
    lengths = torch.randint(0, 13, (rows, C, bins), generator=g).to(torch.uint8).cuda()
    packed = _pack_nibbles_dev(lengths)
    got = native().cachegen_cdf_from_lengths(packed, rows, C, bins)
    assert torch.equal(got.cpu(), cdf_from_lengths(lengths).cpu())
