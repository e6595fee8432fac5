"""Prefill forward with the layer-by-layer direct push hidden under it.

The prefill instance runs a random-init Qwen3-32B tensor-parallel shard
(TP4: 16 of 64 query heads, 2 of 8 KV heads, head_dim 128, MLP 6400 of 25600,
64 layers, hidden 5120) over one 16384-token prompt.  Each layer writes its
rotated K and V into the vLLM paged cache (block 128) registered with this
repo's vLLM connector (``kv_producer``), and the connector's
``save_kv_layer`` launches that layer's push to the decode instance on a side
stream while the forward continues (the decode instance's connector,
``kv_consumer``, reserved its blocks for the request).  With a prefill group
of more than one rank each layer also all-reduces its attention and MLP
outputs over NCCL, as tensor parallelism does.

Reported: forward alone and forward + push, CUDA-event timed on the
prefiller's stream (the push's completion joined into the end event), max
over ranks; the ratio is the cost of pushing during prefill.
"""

from __future__ import annotations

import socket
import time
from types import SimpleNamespace
from typing import Optional

import torch
import torch.nn.functional as F

from .config import LMCacheEngineConfig
from .models.llama import DecoderLayer, LlamaConfig, RMSNorm


def shard_config(tp: int = 4) -> LlamaConfig:
    full = LlamaConfig.qwen3_32b()
    return LlamaConfig(full.vocab_size, full.hidden_size, full.num_layers,
                       full.num_heads // tp, full.num_kv_heads // tp, full.head_dim,
                       full.intermediate_size // tp, full.rope_theta, full.max_position,
                       qk_norm=True)


class ShardPrefill:
    """The forward of one TP shard, writing each layer's KV into ``kv``
    (vLLM layout [2, blocks, block, kv_heads, head_dim] per layer)."""

    def __init__(self, c: LlamaConfig, device, tp_group=None, seed: int = 0):
        torch.manual_seed(seed)
        torch.cuda.manual_seed(seed)
        fk = {"device": device, "dtype": torch.bfloat16}
        self.c = c
        self.layers = [DecoderLayer(c, **fk) for _ in range(c.num_layers)]
        with torch.no_grad():
            for layer in self.layers:
                for p in layer.parameters():
                    if p.dim() == 2:
                        p.normal_(0.0, 0.02)
        half = c.head_dim // 2
        inv = 1.0 / (c.rope_theta ** (torch.arange(half, device=device).float() / half))
        self.inv_freq = inv
        self.tp_group = tp_group

    def _rope(self, x, cos, sin):
        half = self.c.head_dim // 2
        xf = x.float()
        x1, x2 = xf[..., :half], xf[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)

    def _reduce(self, x):
        if self.tp_group is not None:
            torch.distributed.all_reduce(x, group=self.tp_group)
        return x

    @torch.no_grad()
    def forward(self, h: torch.Tensor, kv, slots: torch.Tensor, after_attention=None):
        c = self.c
        T = h.shape[0]
        pos = torch.arange(T, device=h.device).float()
        ang = pos[:, None] * self.inv_freq[None, :]
        cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
        for l, layer in enumerate(self.layers):
            q, k, v = layer.qkv(h)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            kc, vc = kv[l][0], kv[l][1]
            kc.view(-1, c.num_kv_heads * c.head_dim)[slots] = k.reshape(T, -1)
            vc.view(-1, c.num_kv_heads * c.head_dim)[slots] = v.reshape(T, -1)
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                               v.transpose(0, 1)[None], is_causal=True,
                                               enable_gqa=True)
            if after_attention is not None:
                after_attention(l)
            attn = o[0].transpose(0, 1).reshape(T, -1)
            h = h + self._reduce(layer.o_proj(attn))
            x = layer.post_attention_layernorm(h)
            h = h + self._reduce(layer.down_proj(F.silu(layer.gate_proj(x)) * layer.up_proj(x)))
        return h


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(role: str, iport: int, aport: int) -> LMCacheEngineConfig:
    return LMCacheEngineConfig.from_defaults(
        pd_role=role, chunk_size=256, enable_pd=True, transfer_channel="nvlink",
        pd_buffer_device="cuda", pd_buffer_size=8 << 20, local_cpu=False,
        max_local_cpu_size=0.01, pd_peer_host="127.0.0.1", pd_peer_init_port=[iport],
        pd_peer_alloc_port=[aport], pd_backpressure_reserve=0.0, pd_reserve_timeout_s=30.0)


def _sched_out(new=(), scheduled=None):
    cached = SimpleNamespace(req_ids=[], new_token_ids=[], new_block_ids=[],
                             num_computed_tokens=[], resumed_req_ids=set())
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set())


def _bind(worker, meta):
    worker.bind_connector_metadata(meta)
    worker.start_load_kv(None)


def _paged(L, nb, bs, kvh, d, dev):
    return {f"model.layers.{i}.self_attn.attn":
            torch.zeros(2, nb, bs, kvh, d, device=dev, dtype=torch.bfloat16) for i in range(L)}


def run_prefill_overlap(dev, rank: int, world: int, gloo=None, tokens: int = 16384,
                        iters: int = 2, warmup: int = 1, layers: Optional[int] = None) -> dict:
    """Every rank calls this.  N=1: prefiller and decoder in this process
    (loopback push); N>1: ranks < N/2 prefill (one TP group of N/2 ranks),
    rank r + N/2 decodes for rank r."""
    import torch.distributed as dist

    from .integration.vllm.adapter import LMCacheConnectorV1Impl

    c = shard_config(4)
    if layers is not None:
        c.num_layers = layers
    bs, L = 128, c.num_layers
    nb = 2 * ((tokens + bs - 1) // bs)
    pre_role = world == 1 or rank < world // 2
    dec_role = world == 1 or rank >= world // 2
    tp_group = None
    if world > 1:
        members = list(range(world // 2))
        g = dist.new_group(members, backend="nccl")  # every rank creates it
        if pre_role and len(members) > 1:
            tp_group = g
    g0 = torch.Generator().manual_seed(7)
    dblocks = torch.randperm(nb, generator=g0)[: tokens // bs].tolist()
    pblocks = torch.randperm(nb, generator=g0)[: tokens // bs].tolist()
    prompt = list(range(tokens))

    # decode instance first: it binds the ports the prefiller connects to
    dec_w = dec_s = None
    ports = None
    if dec_role:
        iport, aport = _port(), _port()
        dcfg = _cfg("receiver", iport, aport)
        dec_w = LMCacheConnectorV1Impl("worker", dcfg, "Qwen3-32B", bs, world_size=4,
                                       rank=rank % 4, kv_role="kv_consumer")
        dec_w.register_kv_caches(_paged(L, nb, bs, c.num_kv_heads, c.head_dim, dev))
        dec_s = LMCacheConnectorV1Impl("scheduler", dcfg, "Qwen3-32B", bs, world_size=4,
                                       rank=rank % 4, engine=dec_w.engine,
                                       kv_role="kv_consumer")
        ports = (iport, aport)
    if world > 1:
        allp = [None] * world
        dist.all_gather_object(allp, ports, group=gloo)
        ports = allp[rank + world // 2] if pre_role else ports
    model = pre_w = pre_s = kv = None
    if pre_role:
        pcfg = _cfg("sender", *ports)
        pre_w = LMCacheConnectorV1Impl("worker", pcfg, "Qwen3-32B", bs, world_size=4,
                                       rank=rank % 4, kv_role="kv_producer")
        kv = _paged(L, nb, bs, c.num_kv_heads, c.head_dim, dev)
        pre_w.register_kv_caches(kv)
        pre_s = LMCacheConnectorV1Impl("scheduler", pcfg, "Qwen3-32B", bs, world_size=4,
                                       rank=rank % 4, engine=pre_w.engine,
                                       kv_role="kv_producer")
        model = ShardPrefill(c, dev, tp_group, seed=rank)
    t = torch.arange(tokens)
    pslots = (torch.tensor(pblocks)[t // bs] * bs + t % bs).to(dev)
    kv_list = [kv[k] for k in kv] if kv is not None else None
    names = list(kv) if kv is not None else None
    h0 = (torch.randn(tokens, c.hidden_size, device=dev, dtype=torch.bfloat16)
          if pre_role else None)

    def barrier():
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()

    def one(i: int, push: bool) -> float:
        pid = f"ovl-{rank % max(1, world // 2)}-{i}-{int(push)}"
        params = {"lmcache_direct_push": True, "pd_req_id": pid}
        if push and dec_role:
            req = SimpleNamespace(request_id=f"D{i}", prompt_token_ids=prompt,
                                  kv_transfer_params=params)
            need, _ = dec_s.get_num_new_matched_tokens(req, 0)
            dec_s.update_state_after_alloc(req, dblocks, need)
            _bind(dec_w, dec_s.build_connector_meta(_sched_out()))
            dec_w.clear_connector_metadata()
        barrier()  # reservations in place before any prefill starts
        ms = 0.0
        if pre_role:
            if push:
                req = SimpleNamespace(req_id=f"P{i}", prompt_token_ids=prompt,
                                      block_ids=(pblocks,), num_computed_tokens=0,
                                      kv_transfer_params=params)
                meta = pre_s.build_connector_meta(_sched_out([req], scheduled={f"P{i}": tokens}))
                _bind(pre_w, meta)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            model.forward(h0, kv_list, pslots,
                          after_attention=(lambda l: pre_w.save_kv_layer(names[l]))
                          if push else None)
            if push:
                pre_w.wait_for_save()
                pre_w.join_pushes_on_current_stream()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            if push:
                pre_w.clear_connector_metadata()
                pre_s.request_finished(SimpleNamespace(request_id=f"P{i}"), pblocks)
                deadline = time.monotonic() + 30
                while pre_w.get_finished({f"P{i}"})[0] != {f"P{i}"}:
                    if time.monotonic() > deadline:
                        raise RuntimeError("push never reported done")
                    time.sleep(0.001)
        if push and dec_role:
            deadline = time.monotonic() + 30
            while True:
                _, rec = dec_w.get_finished(set())
                if rec:
                    break
                if time.monotonic() > deadline:
                    raise RuntimeError("decoder never received the push")
                time.sleep(0.001)
            if dec_w.get_block_ids_with_load_errors():
                raise RuntimeError("decoder reported load errors")
        barrier()
        return ms

    res = {}
    for push in (False, True):
        for i in range(warmup):
            one(i, push)
        vals = [one(warmup + i, push) for i in range(iters)]
        t_ = torch.tensor([sum(vals) / len(vals)], device=dev)
        if world > 1:
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        res["push" if push else "forward"] = float(t_.item())
    for x in (pre_w, pre_s, dec_w, dec_s):
        if x is not None:
            x.shutdown()
    for x in (pre_w, dec_w):
        if x is not None:
            x.engine.close()
    kv_bytes = tokens * L * 2 * c.num_kv_heads * c.head_dim * 2
    return {"forward_ms": round(res["forward"], 3), "forward_plus_push_ms": round(res["push"], 3),
            "ratio": round(res["push"] / res["forward"], 4), "tokens": tokens, "layers": L,
            "kv_bytes_pushed_per_pair": kv_bytes,
            "model": "Qwen3-32B TP4 shard (16 q heads, 2 KV heads, MLP 6400), random init, "
                     "bf16" + (", NCCL all-reduce per layer in the prefill TP group"
                               if tp_group is not None else ""),
            "path": "vLLM connector kv_producer save_kv_layer -> grant -> per-layer push on a "
                    "side stream; kv_consumer reservation + get_finished",
            "iters": iters, "warmup": warmup}
