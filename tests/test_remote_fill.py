"""RemoteFill session protocol (host side): windowed placement into the
decoder's blocks, replay of lost replies, deadline abort of a dead producer,
refusal and circuit breaking with persistent fallback, admission limits."""

import threading
import time
import uuid

import msgpack
import pytest
import torch
import zmq

from lmcache_ascend_b200.v1.kv_format import PagedKVLayout
from lmcache_ascend_b200.v1.remote_fill import (Admission, CircuitBreaker, CopyDataPlane,
                                                RemoteFillProducer, RemoteFillService,
                                                plan_windows)

from .utils import make_separate_kv, random_slots

L, NB, BS, H, D = 2, 64, 16, 2, 32


def _pair(deadline_s=5.0, slots_for=None):
    src = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    dst = [tuple(torch.zeros_like(t) for t in layer) for layer in src]
    table = {}

    def provider(req_id, n):
        if slots_for is not None:
            return slots_for(req_id, n)
        table[req_id] = random_slots(n, NB * BS, seed=hash(req_id) % 1000)
        return table[req_id]

    svc = RemoteFillService(provider, deadline_s=deadline_s, max_window_tokens=256).start()
    plane = CopyDataPlane(PagedKVLayout(src), PagedKVLayout(dst))
    return src, dst, table, svc, plane


def test_plan_windows():
    assert plan_windows(0, 16, 64) == []
    assert plan_windows(100, 16, 64) == [(0, 64), (64, 100)]
    assert plan_windows(40, 16, 10) == [(0, 16), (16, 32), (32, 40)]  # at least one block


def test_fill_places_every_window_and_finishes():
    src, dst, table, svc, plane = _pair()
    try:
        prod = RemoteFillProducer(svc.url, plane, window_tokens=128, block_size=BS)
        ss = random_slots(600, NB * BS, seed=7)
        res = prod.fill("req-a", ss)
        assert res.ok and res.windows == 5 and res.ready_tokens == 600  # 128-token windows
        assert svc.ready["req-a"] == 600
        ds = table["req-a"]
        for l in range(L):
            for p in range(2):
                a = src[l][p].reshape(NB * BS, -1)[ss]
                b = dst[l][p].reshape(NB * BS, -1)[ds]
                assert torch.equal(a, b)
        prod.close()
    finally:
        svc.stop()


def _raw(url):
    s = zmq.Context.instance().socket(zmq.REQ)
    s.setsockopt(zmq.LINGER, 0)
    s.setsockopt(zmq.RCVTIMEO, 2000)
    s.connect(url)

    def call(op, sid, payload=None, op_id=None):
        s.send(msgpack.packb([op, sid, op_id or uuid.uuid4().hex, payload], use_bin_type=True))
        return msgpack.unpackb(s.recv(), raw=False)
    return s, call


def test_replay_and_deadline_abort_of_a_dead_producer():
    _, _, _, svc, _ = _pair(deadline_s=0.5)
    s, call = _raw(svc.url)
    try:
        st, r = call("OPEN", "", {"req_id": "r1", "num_tokens": 64}, op_id="open-1")
        st2, r2 = call("OPEN", "", {"req_id": "r1", "num_tokens": 64}, op_id="open-1")
        assert st == st2 == "ok" and r == r2 and len(svc.sessions) == 1  # replayed, not re-run
        sid = r["session"]
        call("RESERVE_WINDOW", sid, {"window": 0, "start": 0, "end": 64}, op_id="rw")
        # the producer dies here; the sweep aborts the session after the deadline
        time.sleep(1.2)
        assert svc.aborted.get("r1") == "deadline expired"
        st, r = call("ARM_WINDOW", sid, {"window": 0})
        assert st == "err" and "ABORTED" in r
        assert call("STATUS", sid)[1]["state"] == "ABORTED"
        st, r = call("FINISH", sid)
        assert st == "err"
    finally:
        s.close()
        svc.stop()


def test_refusal_opens_the_circuit_and_falls_back():
    fallbacks = []
    _, _, _, svc, plane = _pair(slots_for=lambda req_id, n: None)  # decoder has no blocks
    try:
        br = CircuitBreaker(threshold=2, ttl_s=0.3)
        prod = RemoteFillProducer(svc.url, plane, breaker=br, fallback=fallbacks.append,
                                  op_timeout_s=1.0)
        for i in range(3):
            res = prod.fill(f"q{i}", torch.arange(32))
            assert not res.ok and res.fell_back
        assert "circuit open" in prod.results[-1].reason  # third attempt skipped the decoder
        assert fallbacks == ["q0", "q1", "q2"]
        time.sleep(0.35)
        assert br.allow(svc.url)  # half-open after the TTL
        prod.close()
    finally:
        svc.stop()


def test_unanswered_decoder_times_out_and_falls_back():
    ctx = zmq.Context.instance()
    dead = ctx.socket(zmq.ROUTER)  # accepts connections, never answers
    dead.setsockopt(zmq.LINGER, 0)
    port = dead.bind_to_random_port("tcp://127.0.0.1")
    got = []
    try:
        prod = RemoteFillProducer(f"tcp://127.0.0.1:{port}", None, op_timeout_s=0.2,
                                  retries=1, fallback=got.append)
        t0 = time.monotonic()
        res = prod.fill("z", torch.arange(16))
        assert not res.ok and got == ["z"] and time.monotonic() - t0 < 3
        prod.close()
    finally:
        dead.close()


def test_admission_bounds_sessions_and_bytes():
    a = Admission(max_sessions=1, max_bytes=100)
    assert a.acquire(500, 0.1)          # oversized request admitted when idle
    assert not a.acquire(1, 0.1)        # session limit
    threading.Timer(0.1, a.release, args=(500,)).start()
    assert a.acquire(60, 1.0)
    a.release(60)


def test_metrics_are_bounded_and_track_sessions():
    """Decoder gauges follow sessions and bytes; producer counters take only
    fixed outcome/reason labels (an unknown reason counts as "other"); the
    admission report and the Prometheus export carry the same numbers."""
    src, dst, table, svc, plane = _pair()
    svc.token_bytes = 2 * L * H * D * 4
    try:
        prod = RemoteFillProducer(svc.url, plane, window_tokens=128, block_size=BS)
        ss = random_slots(300, NB * BS, seed=9)
        assert prod.fill("req-m", ss, nbytes=300 * svc.token_bytes).ok
        snap = svc.metrics_snapshot(publish=True)
        assert snap["active_sessions"] == 0 and snap["active_bytes"] == 0
        assert snap["finished_sessions_total"] == 1
        assert snap["published_bytes_total"] == 300 * svc.token_bytes
        assert snap["reserved_bytes_total"] == 300 * svc.token_bytes
        prod.metrics.outcome("ABORTED", "a reason nobody listed")
        rep = prod.admission_report(publish=True)
        m = rep["metrics"]
        assert m["outcome_LOCAL_FULL"] == 1 and m["reason_other"] == 1
        assert set(k for k in m if k.startswith("reason_")) == \
            {f"reason_{r}" for r in ("none", "circuit_open", "admission_timeout",
                                     "open_rejected", "reservation_rejected", "arm_rejected",
                                     "transfer_failed", "verify_failed", "control_timeout",
                                     "finish_rejected", "other")}
        assert rep["admission"]["admitted_total"] == 1 and rep["admission"]["sessions"] == 0
        try:
            from prometheus_client import REGISTRY

            v = REGISTRY.get_sample_value(
                "lmcache_b200_remote_fill_decoder_finished_sessions_total")
            assert v == 1.0
        except ImportError:
            pass
        prod.close()
    finally:
        svc.stop()


def test_capacity_rejection_is_counted():
    src, dst, table, svc, plane = _pair()
    svc.max_sessions = 0
    try:
        prod = RemoteFillProducer(svc.url, plane, window_tokens=128, block_size=BS)
        res = prod.fill("req-c", random_slots(100, NB * BS, seed=2))
        assert not res.ok
        assert svc.metrics_snapshot()["capacity_rejections_total"] == 1
        assert prod.metrics.snapshot()["reason_open_rejected"] == 1
        prod.close()
    finally:
        svc.stop()
