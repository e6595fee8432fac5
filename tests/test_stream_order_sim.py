"""Stream ordering of the layer-by-layer direct push, on the CPU simulator.

The real ``DirectPrefillPush`` (the prefiller's side-stream push driven from
``save_kv_layer``) runs against a simulated device: the forward's per-layer
KV writes, the push's reads of those rows and its writes into the decoder,
the per-layer flag releases and the decoder's flag waits are deferred
operations executed in random orders that respect stream order and event
waits; writes poison their rows until they complete.  The correct pipeline
passes on every seed; each of four injected faults -- the push does not wait
for the layer's KV write, the ready event is recorded before the write, the
flag is released when the push starts instead of after its writes, and a
corrupted payload -- is caught.
"""

import pytest
import torch

from lmcache_ascend_b200.utils.stream_sim import Sim, SimCuda, Violation
from lmcache_ascend_b200.v1.cache_engine import DirectPrefillPush

L, ROWS, E, T = 4, 64, 8, 24
SEEDS = range(12)


class SimPushBackend:
    """Stands in for the PD backend: one layer push = read the prefiller's
    rows, write them into the decoder's rows, then release the layer flag
    (or, with ``early_flag``, release it as the push starts)."""

    def __init__(self, sim, src, dst, flags, early_flag=False, corrupt=False):
        self.sim, self.src, self.dst, self.flags = sim, src, dst, flags
        self.early_flag, self.corrupt = early_flag, corrupt

    def push_granted_layers(self, src_slots, dst_slots, layer, n, tile):
        s = self.sim.current
        box = {}
        if self.early_flag:
            s.enqueue(lambda: self.flags.__setitem__(layer, self.flags[layer] + 1))
        s.enqueue_read(self.src[layer], src_slots, lambda v: box.__setitem__("v", v),
                       name=f"push read L{layer}")
        bad = self.corrupt and layer == 2
        s.enqueue_write(self.dst[layer], dst_slots,
                        lambda: box["v"] + (1.0 if bad else 0.0), name=f"push write L{layer}")
        if not self.early_flag:
            s.enqueue(lambda: self.flags.__setitem__(layer, self.flags[layer] + 1))


def run(seed, skip_wait=False, early_event=False, early_flag=False, corrupt=False):
    sim = Sim(seed)
    src = [torch.zeros(ROWS, E) for _ in range(L)]
    dst = [torch.zeros(ROWS, E) for _ in range(L)]
    flags = [0] * L
    g = torch.Generator().manual_seed(seed)
    s_slots = torch.randperm(ROWS, generator=g)[:T]
    d_slots = torch.randperm(ROWS, generator=g)[:T]
    kv = [torch.randn(T, E, generator=g) for _ in range(L)]
    seen = {}
    with SimCuda(sim):
        be = SimPushBackend(sim, src, dst, flags, early_flag, corrupt)
        h = DirectPrefillPush.__new__(DirectPrefillPush)
        h.pd, h.req_id, h.src, h.dst = be, "r", s_slots, d_slots
        h.num_tokens, h.num_layers, h.tile_tokens = T, L, 512
        h.pushed, h._done_event, h._finished = 0, None, False
        h.stream = torch.cuda.Stream()
        decoder = torch.cuda.Stream()
        compute = sim.default
        for l in range(L):
            # the forward writes layer l's KV, then save_kv_layer pushes it
            ready = None
            if early_event:
                ready = torch.cuda.Event()
                ready.record(compute)
            compute.enqueue_write(src[l], s_slots, kv[l], name=f"forward L{l}")
            if skip_wait:
                with torch.cuda.stream(h.stream):
                    be.push_granted_layers(h.src, h.dst, l, 1, 512)
            else:
                h.push_layer(l, ready)
            compute.enqueue(lambda: None, name=f"more forward after L{l}")
            # the decoder's attention of layer l waits for the flag, then reads
            decoder.enqueue_cond_wait(lambda l=l: flags[l] >= 1)
            decoder.enqueue_read(dst[l], d_slots, lambda v, l=l: seen.__setitem__(l, v),
                                 name=f"decoder read L{l}")
        h.finish()
        sim.drain()
    sim.check()
    for l in range(L):
        if not torch.equal(seen[l], kv[l]):
            raise Violation(f"layer {l}: decoder read wrong data")


@pytest.mark.parametrize("seed", SEEDS)
def test_direct_push_pipeline_is_ordered(seed):
    run(seed)


@pytest.mark.parametrize("fault", ["skip_wait", "early_event", "early_flag", "corrupt"])
def test_injected_ordering_faults_are_caught(fault):
    caught = 0
    for seed in SEEDS:
        try:
            run(seed, **{fault: True})
        except Violation:
            caught += 1
    assert caught > 0, f"{fault} went unnoticed on every seed"
