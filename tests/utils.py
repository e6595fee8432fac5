"""Shared test helpers: paged KV generators in every supported layout."""

import torch


def make_separate_kv(num_layers, num_blocks, block_size, heads, head_dim, dtype, device,
                     seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(num_layers):
        k = torch.randn(num_blocks, block_size, heads, head_dim, generator=g).to(dtype)
        v = torch.randn(num_blocks, block_size, heads, head_dim, generator=g).to(dtype)
        out.append((k.to(device), v.to(device)))
    return out


def make_merged_kv(num_layers, num_blocks, block_size, heads, head_dim, dtype, device,
                   flashinfer=False, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(num_layers):
        shape = ((num_blocks, 2, block_size, heads, head_dim) if flashinfer else
                 (2, num_blocks, block_size, heads, head_dim))
        out.append(torch.randn(*shape, generator=g).to(dtype).to(device))
    return out


def make_mla_kv(num_layers, num_blocks, block_size, d_lora, d_rope, dtype, device, seed=0,
                flat=False, indexer_dim=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(num_layers):
        if flat:
            out.append(torch.randn(num_blocks, block_size, d_lora + d_rope,
                                   generator=g).to(dtype).to(device))
            continue
        k = torch.randn(num_blocks, block_size, 1, d_lora, generator=g).to(dtype).to(device)
        r = torch.randn(num_blocks, block_size, 1, d_rope, generator=g).to(dtype).to(device)
        if indexer_dim:
            ix = torch.randn(num_blocks, block_size, 1, indexer_dim,
                             generator=g).to(dtype).to(device)
            out.append((k, r, ix))
        else:
            out.append((k, r))
    return out


def zeros_like_kv(kv):
    out = []
    for layer in kv:
        if isinstance(layer, tuple):
            out.append(tuple(torch.zeros_like(t) for t in layer))
        else:
            out.append(torch.zeros_like(layer))
    return out


def random_slots(num_tokens, num_slots, seed=0, device="cpu", dtype=torch.int64):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randperm(num_slots, generator=g)[:num_tokens].to(dtype).to(device)


def block_slots(num_tokens, block_size, num_blocks, seed=0, device="cpu", dtype=torch.int64):
    """vLLM-like slot mapping: a random block table, consecutive slots per block."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    nblk = (num_tokens + block_size - 1) // block_size
    blocks = torch.randperm(num_blocks, generator=g)[:nblk]
    t = torch.arange(num_tokens)
    return (blocks[t // block_size] * block_size + t % block_size).to(dtype).to(device)
