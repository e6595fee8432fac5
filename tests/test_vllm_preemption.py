"""Preemption checkpoints through the vLLM connector roles (CPU tier).

A fake scheduler drives one request through prefill and a few decode steps,
preempts it (vLLM's ``preempted_req_ids``), lets the worker's
``handle_preemptions`` copy the computed KV out before the blocks are reused,
and resumes it on new blocks: the scheduler reports the checkpoint as a
prefix hit and the worker restores it.  Also: a stale generation is
ignored, finished requests cancel their generation, and a TP rank that
cannot restore makes every rank skip the load (agreement) and report the
blocks for recomputation.
"""

from types import SimpleNamespace

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig
from lmcache_ascend_b200.integration.vllm.adapter import LMCacheConnectorV1Impl

L, NB, BS, H, D = 2, 64, 16, 2, 32


def _kv(dev="cpu"):
    return {f"model.layers.{i}.self_attn.attn": torch.zeros(2, NB, BS, H, D, device=dev)
            for i in range(L)}


def _out(new=(), cached=None, scheduled=None, finished=(), preempted=()):
    cached = cached or SimpleNamespace(req_ids=[], new_token_ids=[], new_block_ids=[],
                                       num_computed_tokens=[], resumed_req_ids=set())
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set(finished),
                           preempted_req_ids=set(preempted))


def _slots(blocks, n):
    t = torch.arange(n)
    return torch.tensor(blocks)[t // BS] * BS + t % BS


def _fill(kv, slots, seed):
    g = torch.Generator().manual_seed(seed)
    for x in kv.values():
        x.view(2, NB * BS, -1)[:, slots.to(x.device)] = \
            torch.randn(2, len(slots), H * D, generator=g).to(x.device)


def _read(kv, slots):
    return [x.view(2, NB * BS, -1)[:, slots.to(x.device)].cpu() for x in kv.values()]


def _step(worker, meta):
    worker.bind_connector_metadata(meta)
    worker.handle_preemptions(meta)
    worker.start_load_kv(None)
    for name in worker._layer_names:
        worker.wait_for_layer_load(name)
        worker.save_kv_layer(name, None, None)
    worker.wait_for_save()
    worker.clear_connector_metadata()


def _pair(dev="cpu"):
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.05)
    worker = LMCacheConnectorV1Impl("worker", cfg, "m", BS)
    kv = _kv(dev)
    worker.register_kv_caches(kv)
    sched = LMCacheConnectorV1Impl("scheduler", cfg, "m", BS, engine=worker.engine)
    return sched, worker, kv


def _run_until_preempted(sched, worker, kv, req, blocks):
    """Prefill 150 prompt tokens, decode to 200 tokens, then preempt."""
    sched.on_new_request(req)
    sched.get_num_new_matched_tokens(req, 0)
    sched.update_state_after_alloc(req, None, 0)
    new = SimpleNamespace(req_id=req.request_id, prompt_token_ids=req.prompt_token_ids,
                          block_ids=(blocks,), num_computed_tokens=0)
    _fill(kv, _slots(blocks, 200), seed=1)  # the model's KV for positions 0..199
    _step(worker, sched.build_connector_meta(_out([new], scheduled={req.request_id: 150})))
    req.all_token_ids = list(req.prompt_token_ids) + list(range(9000, 9050))
    cached = SimpleNamespace(req_ids=[req.request_id], new_token_ids=[[]], new_block_ids=[None],
                             num_computed_tokens=[150], resumed_req_ids=set())
    _step(worker, sched.build_connector_meta(_out(cached=cached,
                                                  scheduled={req.request_id: 50})))
    want = _read(kv, _slots(blocks, 200))
    meta = sched.build_connector_meta(_out(preempted=[req.request_id]))
    assert [c["req_id"] for c in meta.preemption_captures] == [req.request_id]
    assert meta.preemption_captures[0]["token_ids"].numel() == 200
    _step(worker, meta)
    return want, meta


@pytest.mark.parametrize("dev", ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)])
def test_preempted_request_resumes_from_its_checkpoint(dev):
    sched, worker, kv = _pair(dev)
    req = SimpleNamespace(request_id="R", prompt_token_ids=list(range(150)))
    blocks = list(range(0, 13))
    want, _ = _run_until_preempted(sched, worker, kv, req, blocks)
    for x in kv.values():
        x.zero_()  # vLLM reuses the freed blocks
    need, _ = sched.get_num_new_matched_tokens(req, 0)
    assert need == 199  # prompt + generated tokens, minus the one vLLM computes
    sched.update_state_after_alloc(req, None, need)
    new_blocks = list(range(20, 33))
    cached = SimpleNamespace(req_ids=["R"], new_token_ids=[[]], new_block_ids=[(new_blocks,)],
                             num_computed_tokens=[0], resumed_req_ids={"R"})
    meta = sched.build_connector_meta(_out(cached=cached, scheduled={"R": 1}))
    assert meta.requests and meta.requests[0].load_spec is not None
    _step(worker, meta)
    if dev == "cuda":
        torch.cuda.synchronize()
    got = _read(kv, _slots(new_blocks, 200))
    for a, b in zip(want, got):
        assert torch.equal(a, b)
    # finishing the request cancels its checkpoint generation
    meta = sched.build_connector_meta(_out(finished=["R"]))
    assert meta.preemption_cancels == [("R", 1)]
    worker.shutdown()
    worker.engine.close()


def test_stale_generation_is_ignored():
    sched, worker, kv = _pair()
    req = SimpleNamespace(request_id="S", prompt_token_ids=list(range(150)))
    _, meta1 = _run_until_preempted(sched, worker, kv, req, list(range(0, 13)))
    ck = worker.checkpointer
    n_results = len(ck.results)
    stale = dict(meta1.preemption_captures[0])
    # a newer generation supersedes: replaying generation 1 after generation 2
    ck.capture("S", 2, stale["token_ids"].tolist(), stale["slot_mapping"])
    assert ck.capture("S", 1, stale["token_ids"].tolist(), stale["slot_mapping"]) == 0
    assert ck.seal("S", 1, stale["token_ids"].tolist()) is None
    assert len(ck.results) == n_results
    ck.cancel("S")
    worker.shutdown()
    worker.engine.close()


def test_tp_disagreement_skips_the_load_on_every_rank():
    sched, worker, kv = _pair()
    req = SimpleNamespace(request_id="T", prompt_token_ids=list(range(150)))
    _run_until_preempted(sched, worker, kv, req, list(range(0, 13)))
    for x in kv.values():
        x.fill_(7.0)
    # another TP rank could not capture: the all-true collective says no
    worker.engine.collective_all_true_fn = lambda ok: False
    need, _ = sched.get_num_new_matched_tokens(req, 0)
    sched.update_state_after_alloc(req, None, need)
    new_blocks = list(range(40, 53))
    cached = SimpleNamespace(req_ids=["T"], new_token_ids=[[]], new_block_ids=[(new_blocks,)],
                             num_computed_tokens=[0], resumed_req_ids={"T"})
    _step(worker, sched.build_connector_meta(_out(cached=cached, scheduled={"T": 1})))
    got = _read(kv, _slots(new_blocks, 199))
    assert all(bool((g == 7.0).all()) for g in got)  # nothing was loaded
    bad = worker.get_block_ids_with_load_errors()
    assert bad and set(bad) <= set(new_blocks)
    worker.shutdown()
    worker.engine.close()
