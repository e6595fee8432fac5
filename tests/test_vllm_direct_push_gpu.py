"""Direct paged push through the vLLM connector roles, with the real kernels.

The prefill instance's worker pushes each layer from ``save_kv_layer`` on a
side stream behind that layer's KV write; the decode instance's worker
reserved its blocks and reports the request received once every layer's
flag arrived.  The decoder's paged cache is compared byte for byte with the
prefiller's rows.  One GPU: both instances in one process (loopback, same
kernels, local addresses).  Two GPUs: one process per instance (spawn),
NVLink peer stores; skipped with fewer GPUs.
"""

import os
import socket
import time
import traceback
from types import SimpleNamespace

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
L, NB, BS, H, D = 4, 64, 128, 2, 128
PROMPT = list(range(1000, 1000 + 1500))
PARAMS = {"lmcache_direct_push": True, "pd_req_id": "job-42"}
DBLOCKS = list(range(40, 52))
PBLOCKS = list(range(3, 15))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _sched_out(new=(), scheduled=None):
    cached = SimpleNamespace(req_ids=[], new_token_ids=[], new_block_ids=[],
                             num_computed_tokens=[], resumed_req_ids=set())
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set())


def _cfg(role, iport, aport):
    from lmcache_ascend_b200.config import LMCacheEngineConfig

    return LMCacheEngineConfig.from_defaults(
        pd_role=role, chunk_size=256, enable_pd=True, transfer_channel="nvlink",
        pd_buffer_device="cuda", pd_buffer_size=8 << 20, local_cpu=False,
        max_local_cpu_size=0.01, pd_peer_host="127.0.0.1", pd_peer_init_port=[iport],
        pd_peer_alloc_port=[aport], pd_backpressure_reserve=0.0, pd_reserve_timeout_s=10.0)


def _kv(dev, seed):
    g = torch.Generator().manual_seed(seed)
    return {f"model.layers.{i}.self_attn.attn":
            torch.randn(2, NB, BS, H, D, generator=g).to(torch.bfloat16).to(dev)
            for i in range(L)}


def _rows(kv, blocks, n):
    t = torch.arange(n)
    slots = (torch.tensor(blocks)[t // BS] * BS + t % BS).to(next(iter(kv.values())).device)
    return [x.view(2, NB * BS, -1)[:, slots].cpu() for x in kv.values()]


def _forward(worker, meta, on_layer=None):
    worker.bind_connector_metadata(meta)
    worker.start_load_kv(None)
    for i, name in enumerate(worker._layer_names):
        worker.wait_for_layer_load(name)
        if on_layer is not None:
            on_layer(i)
        worker.save_kv_layer(name, None, None)
    worker.wait_for_save()
    worker.clear_connector_metadata()


def _decoder(dev, iport, aport):
    from lmcache_ascend_b200.integration.vllm.adapter import LMCacheConnectorV1Impl

    cfg = _cfg("receiver", iport, aport)
    kv = {k: torch.zeros_like(v) for k, v in _kv(dev, 0).items()}
    w = LMCacheConnectorV1Impl("worker", cfg, "m", BS, kv_role="kv_consumer")
    w.register_kv_caches(kv)
    s = LMCacheConnectorV1Impl("scheduler", cfg, "m", BS, engine=w.engine,
                               kv_role="kv_consumer")
    req = SimpleNamespace(request_id="D1", prompt_token_ids=PROMPT, kv_transfer_params=PARAMS)
    assert s.get_num_new_matched_tokens(req, 0) == (len(PROMPT) - 1, True)
    s.update_state_after_alloc(req, DBLOCKS, len(PROMPT) - 1)
    _forward(w, s.build_connector_meta(_sched_out()))
    return w, s, kv


def _prefiller(dev, iport, aport, kv_src):
    from lmcache_ascend_b200.integration.vllm.adapter import LMCacheConnectorV1Impl

    cfg = _cfg("sender", iport, aport)
    w = LMCacheConnectorV1Impl("worker", cfg, "m", BS, kv_role="kv_producer")
    kv = {k: torch.zeros_like(v) for k, v in kv_src.items()}
    w.register_kv_caches(kv)
    s = LMCacheConnectorV1Impl("scheduler", cfg, "m", BS, engine=w.engine,
                               kv_role="kv_producer")
    req = SimpleNamespace(req_id="P1", prompt_token_ids=PROMPT, block_ids=(PBLOCKS,),
                          num_computed_tokens=0, kv_transfer_params=PARAMS)
    meta = s.build_connector_meta(_sched_out([req], scheduled={"P1": len(PROMPT)}))
    names = list(kv)

    def write_layer(i):  # "the model's forward wrote layer i's KV" (on the current stream)
        kv[names[i]].copy_(kv_src[names[i]])

    _forward(w, meta, on_layer=write_layer)
    assert s.request_finished(SimpleNamespace(request_id="P1"), PBLOCKS) == (True, None)
    deadline = time.monotonic() + 20
    while True:
        sending, _ = w.get_finished({"P1"})
        if sending == {"P1"} or time.monotonic() > deadline:
            break
        time.sleep(0.005)
    assert sending == {"P1"}
    return w, s, kv


def _wait_received(w):
    deadline = time.monotonic() + 20
    while time.monotonic() < deadline:
        _, recving = w.get_finished(set())
        if recving:
            return recving
        time.sleep(0.005)
    return None


def test_direct_push_connector_roles_one_gpu():
    dev = torch.device("cuda", 0)
    iport, aport = _port(), _port()
    dw, ds, dkv = _decoder(dev, iport, aport)
    kv_src = _kv(dev, 1)
    pw, ps, pkv = _prefiller(dev, iport, aport, kv_src)
    try:
        assert _wait_received(dw) == {"D1"}
        assert not dw.get_block_ids_with_load_errors()
        n = len(PROMPT) - 1
        for a, b in zip(_rows(pkv, PBLOCKS, n), _rows(dkv, DBLOCKS, n)):
            assert torch.equal(a, b)
    finally:
        for x in (pw, ps, dw, ds):
            x.shutdown()
        pw.engine.close()
        dw.engine.close()


def _dec_proc(iport, aport, q):
    try:
        dev = torch.device("cuda", 1)
        torch.cuda.set_device(dev)
        w, s, kv = _decoder(dev, iport, aport)
        q.put(("reserved", None))
        got = _wait_received(w)
        rows = _rows(kv, DBLOCKS, len(PROMPT) - 1)
        q.put(("decoder", (got == {"D1"}, [r for r in rows])))
        time.sleep(1.0)
        w.shutdown()
        s.shutdown()
        w.engine.close()
    except Exception:
        q.put(("decoder", (False, traceback.format_exc())))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_direct_push_connector_roles_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    iport, aport = _port(), _port()
    p = ctx.Process(target=_dec_proc, args=(iport, aport, q))
    p.start()
    try:
        tag, _ = q.get(timeout=120)
        assert tag == "reserved"
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        kv_src = _kv(dev, 1)
        pw, ps, pkv = _prefiller(dev, iport, aport, kv_src)
        tag, (ok, rows) = q.get(timeout=120)
        assert ok, rows
        for a, b in zip(_rows(pkv, PBLOCKS, len(PROMPT) - 1), rows):
            assert torch.equal(a, b)
        pw.shutdown()
        ps.shutdown()
        pw.engine.close()
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
