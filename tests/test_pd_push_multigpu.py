"""K9 across two GPUs: sender (GPU 0) pushes into the receiver's (GPU 1)
paged cache over NVLink through CUDA IPC peer mappings; verified byte-exact
on the receiver.  Two processes (spawn), descriptors exchanged through a
multiprocessing queue.  All waits are bounded; a child that fails reports it
through the queue and exits."""

import os
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

L, NB, BS, H, D, T = 8, 64, 128, 2, 128, 4096


def _cache(seed, dev):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(NB, BS, H, D, generator=g).to(torch.bfloat16).to(dev),
             torch.randn(NB, BS, H, D, generator=g).to(torch.bfloat16).to(dev))
            for _ in range(L)]


def _slots(seed):
    g = torch.Generator().manual_seed(seed)
    blocks = torch.randperm(NB, generator=g)[: T // BS]
    t = torch.arange(T)
    return (blocks[t // BS] * BS + t % BS).to(torch.int32)


def _receiver(q_desc, q_done, q_res):
    try:
        from lmcache_ascend_b200.parallel.pd_push import PushReceiver
        from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

        dev = torch.device("cuda", 1)
        torch.cuda.set_device(dev)
        dst = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in _cache(0, dev)]
        recv = PushReceiver(PagedKVLayout(dst))
        q_desc.put(recv.desc.to_dict())
        tg = recv.expect(T)
        recv.wait(tg, timeout_s=10.0)
        torch.cuda.synchronize()
        st = recv.status.read()
        ok = st["code"] == 0
        if ok:
            src = _cache(1, "cpu")
            ds = _slots(22).long()
            for (k, v), (k2, v2) in zip(src, dst):
                ok &= torch.equal(k.view(-1, H * D)[_slots(11).long()],
                                  k2.cpu().view(-1, H * D)[ds])
                ok &= torch.equal(v.view(-1, H * D)[_slots(11).long()],
                                  v2.cpu().view(-1, H * D)[ds])
        q_done.get(timeout=60)  # keep mappings alive until the sender closed them
        q_res.put(("receiver", bool(ok), st))
    except Exception:
        q_res.put(("receiver", False, traceback.format_exc()))


def _sender(q_desc, q_done, q_res):
    try:
        from lmcache_ascend_b200.parallel.pd_push import PushSender, ReceiverDesc
        from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        src = _cache(1, dev)
        send = PushSender(PagedKVLayout(src))
        send.connect([ReceiverDesc.from_dict(q_desc.get(timeout=60))])
        send.push(_slots(11).to(dev), _slots(22).to(dev))
        torch.cuda.synchronize()
        st = send.status.read()
        send.close()
        q_done.put(True)
        q_res.put(("sender", st["code"] == 0, st))
    except Exception:
        q_done.put(True)
        q_res.put(("sender", False, traceback.format_exc()))


def test_push_two_gpus():
    ctx = mp.get_context("spawn")
    q_desc, q_done, q_res = ctx.Queue(), ctx.Queue(), ctx.Queue()
    pr = ctx.Process(target=_receiver, args=(q_desc, q_done, q_res))
    ps = ctx.Process(target=_sender, args=(q_desc, q_done, q_res))
    pr.start()
    ps.start()
    res = [q_res.get(timeout=180) for _ in range(2)]
    ps.join(60)
    pr.join(60)
    for who, ok, info in res:
        assert ok, f"{who}: {info}"
