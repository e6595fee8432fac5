"""vLLM connector roles for the direct paged push, on the host.

A prefill instance (``kv_producer``) and a decode instance (``kv_consumer``)
each run the connector's scheduler and worker logic with light stand-ins for
vLLM's objects; the router gives both the same ``pd_req_id``.  The push
launcher and the decoder's flag receiver are fakes recording what would run
on the GPU (the byte-exact 2-GPU version is ``test_vllm_direct_push_gpu``).
Checks: the decoder reports an asynchronous external hit and reserves the
blocks vLLM allocated; the prefiller's first ``save_kv_layer`` gets the
grant (the decoder's slots come back in it) and every layer launches once,
in layer order, after the grant; vLLM keeps the prefiller's blocks
(``request_finished`` -> True) until ``get_finished`` reports the push done;
the decoder reports the request received.  A decoder that never reserved
gets no launch at all.
"""

import socket
from types import SimpleNamespace

import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig
from lmcache_ascend_b200.integration.vllm.adapter import LMCacheConnectorV1Impl

from .test_pd_direct_handshake import FakeReceiver, FakeSender

L, NB, BS, H, D = 3, 64, 16, 2, 32


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _kv():
    return {f"model.layers.{i}.self_attn.attn": torch.zeros(2, NB, BS, H, D) for i in range(L)}


def _sched_out(new=(), scheduled=None, finished=()):
    cached = SimpleNamespace(req_ids=[], new_token_ids=[], new_block_ids=[],
                             num_computed_tokens=[], resumed_req_ids=set())
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set(finished))


def _instances(iport, aport, reserve_timeout=2.0):
    base = dict(chunk_size=64, enable_pd=True, transfer_channel="tcp", pd_buffer_device="cpu",
                pd_buffer_size=1 << 20, local_cpu=False, max_local_cpu_size=0.01,
                pd_peer_host="127.0.0.1", pd_peer_init_port=[iport],
                pd_peer_alloc_port=[aport], pd_backpressure_reserve=0.0,
                pd_reserve_timeout_s=reserve_timeout, blocking_timeout_secs=2.0)
    dcfg = LMCacheEngineConfig.from_defaults(pd_role="receiver", **base)
    dec = LMCacheConnectorV1Impl("worker", dcfg, "m", BS, kv_role="kv_consumer")
    dec.register_kv_caches(_kv())
    pd_r = dec.engine.storage_manager.backends["PDBackend"]
    pd_r.push_receiver = FakeReceiver(dec.engine.gpu_connector.layout)
    dec_s = LMCacheConnectorV1Impl("scheduler", dcfg, "m", BS, engine=dec.engine,
                                   kv_role="kv_consumer")
    pcfg = LMCacheEngineConfig.from_defaults(pd_role="sender", **base)
    pre = LMCacheConnectorV1Impl("worker", pcfg, "m", BS, kv_role="kv_producer")
    pre.register_kv_caches(_kv())
    pd_s = pre.engine.storage_manager.backends["PDBackend"]
    pd_s.push_sender = FakeSender(pre.engine.gpu_connector.layout)
    pre_s = LMCacheConnectorV1Impl("scheduler", pcfg, "m", BS, engine=pre.engine,
                                   kv_role="kv_producer")
    return dec, dec_s, pre, pre_s, pd_r, pd_s


def _forward(worker, meta):
    worker.bind_connector_metadata(meta)
    worker.start_load_kv(None)
    for name in worker._layer_names:
        worker.wait_for_layer_load(name)
        worker.save_kv_layer(name, None, None)
    worker.wait_for_save()
    worker.clear_connector_metadata()


def _close(*impls):
    for i in impls:
        i.shutdown()
        if i.role == "worker":
            i.engine.close()


def test_direct_push_through_connector_roles():
    dec, dec_s, pre, pre_s, pd_r, pd_s = _instances(_port(), _port())
    try:
        prompt = list(range(500, 800))  # 300 tokens
        params = {"lmcache_direct_push": True, "pd_req_id": "job-7"}
        # --- decoder scheduler: async external hit, blocks, reservation
        dreq = SimpleNamespace(request_id="D1", prompt_token_ids=prompt,
                               kv_transfer_params=params)
        assert dec_s.get_num_new_matched_tokens(dreq, 0) == (299, True)
        dblocks = list(range(30, 49))
        dec_s.update_state_after_alloc(dreq, dblocks, 299)
        dmeta = dec_s.build_connector_meta(_sched_out())
        assert [r.direct["mode"] for r in dmeta.requests] == ["recv"]
        _forward(dec, dmeta)
        assert "job-7" in pd_r.reservations
        assert dec.get_finished(set()) == (None, None)  # nothing granted yet
        # --- prefiller: the whole prompt in one step
        pblocks = list(range(0, 19))
        preq = SimpleNamespace(req_id="P1", prompt_token_ids=prompt, block_ids=(pblocks,),
                               num_computed_tokens=0, kv_transfer_params=params)
        pmeta = pre_s.build_connector_meta(_sched_out([preq], scheduled={"P1": 300}))
        assert [r.direct["mode"] for r in pmeta.requests] == ["send"]
        _forward(pre, pmeta)
        launches = pd_s.push_sender.launches
        assert [(lb, nl) for _, _, lb, nl in launches] == [(l, 1) for l in range(L)]
        src, dst = launches[0][0].long(), launches[0][1].long()
        t = torch.arange(299)
        assert torch.equal(dst, torch.tensor(dblocks)[t // BS] * BS + t % BS)
        assert torch.equal(src, torch.tensor(pblocks)[t // BS] * BS + t % BS)
        # vLLM holds the prefiller's blocks until the push is reported done
        assert pre_s.request_finished(SimpleNamespace(request_id="P1"), pblocks) == (True, None)
        sending, _ = pre.get_finished({"P1"})
        assert sending == {"P1"}
        _, recving = dec.get_finished(set())
        assert recving == {"D1"}
        assert pd_r.push_receiver.waits  # the per-layer flag wait was enqueued
    finally:
        _close(dec, dec_s, pre, pre_s)


def test_unreserved_request_gets_no_launch():
    dec, dec_s, pre, pre_s, pd_r, pd_s = _instances(_port(), _port(), reserve_timeout=0.2)
    try:
        prompt = list(range(100))
        params = {"lmcache_direct_push": True, "pd_req_id": "job-unknown"}
        preq = SimpleNamespace(req_id="P2", prompt_token_ids=prompt, block_ids=([0, 1, 2, 3,
                                                                                 4, 5, 6],),
                               num_computed_tokens=0, kv_transfer_params=params)
        pmeta = pre_s.build_connector_meta(_sched_out([preq], scheduled={"P2": 100}))
        _forward(pre, pmeta)
        assert pd_s.push_sender.launches == []
        assert pre_s.request_finished(SimpleNamespace(request_id="P2"), []) == (True, None)
        sending, _ = pre.get_finished({"P2"})
        assert sending == {"P2"}  # the blocks are released again
    finally:
        _close(dec, dec_s, pre, pre_s)
