"""NVLS fan-out: one prefiller pushes through the multicast staging buffer,
every other member receives the rows, and back-to-back pushes wait for the
members' staging release (2+ GPUs; skipped otherwise, and where the system
has no NVLink multicast)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, NB, BS, H, D, T = 4, 32, 128, 2, 128, 1500


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from lmcache_ascend_b200.parallel.pd_multicast import MulticastFanout
    from lmcache_ascend_b200.v1.kv_format import PagedKVLayout
    from tests.utils import block_slots, make_separate_kv

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, dev, seed=1)  # same on all ranks
        dst = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, dev, seed=2 + rank)
        ss = block_slots(T, BS, NB, seed=3, device=dev, dtype=torch.int32)
        ds = block_slots(T, BS, NB, seed=4 + rank, device=dev, dtype=torch.int32)
        fan = MulticastFanout(dist.group.WORLD, L, 2, H * D * 2, 2048, dev)
        if not fan.has_multicast:
            q.put((rank, "no-multicast"))
            return
        def same():
            return all(torch.equal(src[l][p].view(NB * BS, -1)[ss.long()],
                                   dst[l][p].view(NB * BS, -1)[ds.long()])
                       for l in range(L) for p in range(2))

        tg = fan.expect(T)
        if rank == 0:
            fan.push(PagedKVLayout(src), ss)
        fan.wait(tg, timeout_s=5.0)
        fan.scatter(PagedKVLayout(dst), ds, T)
        torch.cuda.synchronize()
        fan.check()
        ok = same()
        # second push, consumed two layers at a time as each pair lands
        for l in range(L):
            for p in range(2):
                dst[l][p].zero_()
        dist.barrier()
        tg = fan.expect(T)
        if rank == 0:
            fan.push(PagedKVLayout(src), ss)
        for l0 in range(0, L, 2):
            fan.wait(tg[l0:l0 + 2], timeout_s=5.0, layer_begin=l0)
            fan.scatter(PagedKVLayout(dst), ds, T, layer_begin=l0, num_layers=2)
        torch.cuda.synchronize()
        fan.check()
        ok = ok and same()
        # pushes 3 and 4 with new rows and no host barrier in between: the
        # root's push waits (on its stream, bounded) until every member
        # released the previous push through the root's release counter
        for seed in (5, 6):
            src = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, dev, seed=seed)
            tg = fan.expect(T)
            if rank == 0:
                fan.push(PagedKVLayout(src), ss, release_timeout_s=5.0)
            fan.wait(tg, timeout_s=5.0)
            fan.scatter(PagedKVLayout(dst), ds, T)
            torch.cuda.synchronize()
            fan.check()
            ok = ok and same()
        dist.barrier()
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multicast_fanout_every_member_receives():
    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    if all(v == "no-multicast" for v in res.values()):
        pytest.skip("no NVLink multicast on this system")
    assert all(v == "ok" for v in res.values()), res
