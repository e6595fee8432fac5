"""RemoteFill with the NVLink push kernel as data plane and per-layer flag
verification on the decoder (loopback on one GPU: same kernel, local
addresses)."""

import pytest
import torch

from lmcache_ascend_b200.parallel.pd_push import PushReceiver, PushSender
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout
from lmcache_ascend_b200.v1.remote_fill import PushDataPlane, RemoteFillProducer, RemoteFillService
from lmcache_ascend_b200.v1.remote_fill.decoder import PushVerifier

from .utils import block_slots, make_separate_kv

pytestmark = pytest.mark.gpu


def test_remote_fill_over_push_kernel():
    L, NB, BS, H, D = 4, 64, 128, 2, 128
    src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=1)
    dst = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=2)
    recv = PushReceiver(PagedKVLayout(dst))
    send = PushSender(PagedKVLayout(src), engine="auto")
    send.connect([recv.desc])
    T = 1500
    ds = block_slots(T, BS, NB, seed=3, device="cuda")
    svc = RemoteFillService(lambda r, n: ds[:n], verifier=PushVerifier(recv, 128, 2.0),
                            max_window_tokens=512).start()
    try:
        prod = RemoteFillProducer(svc.url, PushDataPlane(send, 128), window_tokens=512,
                                  block_size=BS)
        ss = block_slots(T, BS, NB, seed=4, device="cuda")
        res = prod.fill("req", ss)
        assert res.ok and res.windows == 3 and svc.ready["req"] == T
        torch.cuda.synchronize()
        for l in range(L):
            for p in range(2):
                a = src[l][p].view(NB * BS, -1)[ss.long()]
                b = dst[l][p].view(NB * BS, -1)[ds.long()]
                assert torch.equal(a, b)
        send.check()
        recv.check()
        prod.close()
    finally:
        svc.stop()
        send.close()
