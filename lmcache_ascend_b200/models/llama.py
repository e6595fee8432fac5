"""Compact Llama / Qwen3 decoder for CacheBlend and end-to-end tests.

Pure PyTorch, random init (no checkpoints on this machine), with the pieces
the blender needs: per-layer Q/K/V projection (Qwen3 adds per-head q/k RMS
norm), neox RoPE from a vLLM-layout cos/sin cache, causal attention by
position (so a subset of query tokens can attend to the full key set), and
writes of each layer's rotated K and V into a vLLM paged cache (SEPARATE_KV
per layer: (K, V) [num_blocks, block_size, kv_heads, head_dim]).

This is the model side of the reference's blend wrappers
(lmcache_ascend/v1/blend/models/llama.py, qwen3.py, models.py), which wrap
vLLM's model; here the model is self-contained so blending runs without a
serving engine.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Generator, List, Optional

import torch
import torch.nn.functional as F
from torch import nn

from ..ops.reference import make_cos_sin_cache


@dataclass
class LlamaConfig:
    vocab_size: int = 32000
    hidden_size: int = 256
    num_layers: int = 4
    num_heads: int = 8
    num_kv_heads: int = 2
    head_dim: int = 32
    intermediate_size: int = 512
    rope_theta: float = 10000.0
    max_position: int = 8192
    rms_eps: float = 1e-6
    qk_norm: bool = False  # Qwen3

    @staticmethod
    def tiny(**kw) -> "LlamaConfig":
        return LlamaConfig(**kw)

    @staticmethod
    def llama3_8b() -> "LlamaConfig":
        return LlamaConfig(128256, 4096, 32, 32, 8, 128, 14336, 500000.0, 131072)

    @staticmethod
    def qwen3_32b() -> "LlamaConfig":
        return LlamaConfig(151936, 5120, 64, 64, 8, 128, 25600, 1000000.0, 40960, qk_norm=True)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, **fk):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, **fk))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


class DecoderLayer(nn.Module):
    def __init__(self, c: LlamaConfig, **fk):
        super().__init__()
        self.c = c
        H, KH, D, E = c.num_heads, c.num_kv_heads, c.head_dim, c.hidden_size
        self.input_layernorm = RMSNorm(E, c.rms_eps, **fk)
        self.q_proj = nn.Linear(E, H * D, bias=False, **fk)
        self.k_proj = nn.Linear(E, KH * D, bias=False, **fk)
        self.v_proj = nn.Linear(E, KH * D, bias=False, **fk)
        self.o_proj = nn.Linear(H * D, E, bias=False, **fk)
        self.q_norm = RMSNorm(D, c.rms_eps, **fk) if c.qk_norm else None
        self.k_norm = RMSNorm(D, c.rms_eps, **fk) if c.qk_norm else None
        self.post_attention_layernorm = RMSNorm(E, c.rms_eps, **fk)
        self.gate_proj = nn.Linear(E, c.intermediate_size, bias=False, **fk)
        self.up_proj = nn.Linear(E, c.intermediate_size, bias=False, **fk)
        self.down_proj = nn.Linear(c.intermediate_size, E, bias=False, **fk)

    def qkv(self, hidden):
        c = self.c
        x = self.input_layernorm(hidden)
        q = self.q_proj(x).view(-1, c.num_heads, c.head_dim)
        k = self.k_proj(x).view(-1, c.num_kv_heads, c.head_dim)
        v = self.v_proj(x).view(-1, c.num_kv_heads, c.head_dim)
        if self.q_norm is not None:
            q, k = self.q_norm(q), self.k_norm(k)
        return q, k, v

    def post(self, residual, attn_out):
        h = residual + self.o_proj(attn_out)
        x = self.post_attention_layernorm(h)
        return h + self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LlamaForBlend(nn.Module):
    def __init__(self, config: LlamaConfig, device="cpu", dtype=torch.float32, seed: int = 0,
                 lm_head: bool = False):
        """Parameters are created on ``device`` in ``dtype`` (a 32B model is
        built on the GPU directly) and drawn from N(0, 0.05^2)."""
        super().__init__()
        torch.manual_seed(seed)
        if torch.device(device).type == "cuda":
            torch.cuda.manual_seed(seed)
        fk = {"device": device, "dtype": dtype}
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, **fk)
        self.layers = nn.ModuleList([DecoderLayer(config, **fk)
                                     for _ in range(config.num_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_eps, **fk)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False, **fk) \
            if lm_head else None
        with torch.no_grad():
            for p in self.parameters():
                if p.dim() == 2:
                    p.normal_(0.0, 0.05)
        self.cos_sin_cache = make_cos_sin_cache(config.max_position, config.head_dim,
                                                config.rope_theta).to(device)
        self.is_neox_style = True
        self.head_size = config.head_dim
        self.device = torch.device(device)
        self.dtype = dtype

    # ---------------------------------------------------------------- rope
    def rope(self, positions: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """neox RoPE of x [T, heads, D] at ``positions`` (fp32 math)."""
        half = self.config.head_dim // 2
        cs = self.cos_sin_cache[positions.long()].float()
        cos, sin = cs[:, None, :half], cs[:, None, half:]
        xf = x.float()
        x1, x2 = xf[..., :half], xf[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)

    def rotary_emb(self, positions, q, k):
        return self.rope(positions, q), self.rope(positions, k)

    # ----------------------------------------------------------- attention
    def attend(self, q, k, v, q_pos, k_pos):
        """q [Tq, H, D] at q_pos; k, v [Tk, KH, D] at k_pos; causal by position."""
        c = self.config
        rep = c.num_heads // c.num_kv_heads
        kk = k.repeat_interleave(rep, dim=1)
        vv = v.repeat_interleave(rep, dim=1)
        mask = q_pos[:, None] >= k_pos[None, :]
        o = F.scaled_dot_product_attention(q.transpose(0, 1), kk.transpose(0, 1),
                                           vv.transpose(0, 1), attn_mask=mask[None])
        return o.transpose(0, 1).reshape(q.shape[0], -1)

    @staticmethod
    def write_kv(kv_layer, slot_mapping, k, v):
        kc, vc = kv_layer
        kc.view(-1, kc.shape[-2] * kc.shape[-1])[slot_mapping.long()] = \
            k.reshape(k.shape[0], -1).to(kc.dtype)
        vc.view(-1, vc.shape[-2] * vc.shape[-1])[slot_mapping.long()] = \
            v.reshape(v.shape[0], -1).to(vc.dtype)

    # ------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, kv_caches: List, slot_mapping: torch.Tensor,
                positions: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Full forward; writes every layer's rotated K and V into the paged cache."""
        tokens = tokens.to(self.device)
        pos = positions.to(self.device) if positions is not None else \
            torch.arange(tokens.numel(), device=self.device)
        h = self.embed_tokens(tokens)
        for l, layer in enumerate(self.layers):
            q, k, v = layer.qkv(h)
            q, k = self.rotary_emb(pos, q, k)
            self.write_kv(kv_caches[l], slot_mapping, k, v)
            h = layer.post(h, self.attend(q, k, v, pos, pos))
        return self.norm(h)

    # ------------------------------------------------ decode on cached KV
    @torch.no_grad()
    def decode_step(self, token: torch.Tensor, position: int, kv_caches: List,
                    ctx_slots: torch.Tensor, new_slot: torch.Tensor,
                    before_layer=None) -> torch.Tensor:
        """One token at ``position`` attending to the cached context (paged
        slots ``ctx_slots`` of positions 0..position-1) and to itself; writes
        its K/V at ``new_slot`` and returns the greedy next-token id (device
        int64 [1]).  ``before_layer(l)`` runs before layer l reads its cache
        (a layerwise KV load hooks in there)."""
        c = self.config
        h = self.embed_tokens(token.to(self.device).view(1))
        pos = torch.full((1,), position, device=self.device, dtype=torch.long)
        slots = torch.cat([ctx_slots.to(self.device).long(), new_slot.to(self.device).view(1).long()])
        for l, layer in enumerate(self.layers):
            if before_layer is not None:
                before_layer(l)
            q, k, v = layer.qkv(h)
            q, k = self.rotary_emb(pos, q, k)
            self.write_kv(kv_caches[l], new_slot.view(1), k, v)
            kc, vc = kv_caches[l]
            K = kc.view(-1, c.num_kv_heads, c.head_dim).index_select(0, slots)
            V = vc.view(-1, c.num_kv_heads, c.head_dim).index_select(0, slots)
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], K.transpose(0, 1)[None],
                                               V.transpose(0, 1)[None], enable_gqa=True)
            h = layer.post(h, o[0].transpose(0, 1).reshape(1, -1))
        hs = self.norm(h)
        if self.lm_head is None:
            return hs
        return self.lm_head(hs).argmax(dim=-1)

    # --------------------------------------------------- layerwise blending
    @torch.no_grad()
    def compute_layer(self, tokens: torch.Tensor, blender, kv_caches: List,
                      slot_mapping: torch.Tensor) -> Generator[None, None, torch.Tensor]:
        """Layer-by-layer forward driven by the blender: at each layer the
        blender sees fresh Q/K/V (after RoPE), may narrow the query set to the
        tokens to recompute, and returns the keys/values to attend to (cached
        KV with recomputed rows merged in).  The merged KV is written back to
        the paged cache.  Yields once per layer."""
        tokens = tokens.to(self.device)
        n = tokens.numel()
        all_pos = torch.arange(n, device=self.device)
        h = self.embed_tokens(tokens)
        for l, layer in enumerate(self.layers):
            q, k, v = layer.qkv(h)
            q, k, v, h, _ = blender.process_qkv(q, k, v, h, l, self)
            q_pos = blender.metadata.positions
            self.write_kv(kv_caches[l], slot_mapping, k, v)
            h = layer.post(h, self.attend(q, k, v, q_pos, all_pos))
            yield
        return self.norm(h)
