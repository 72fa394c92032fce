"""Seeded synthetic inputs of the BASELINE configurations, as plain tensors.

Shared by ``bench.py`` (both arms), the microbenchmarks and the parity tests,
so that every one of them sees the same numbers for the same seed.  Nothing
here calls a kernel.
"""

from __future__ import annotations

import math

import torch


def workload_lens(seed: int, batch: int = 64, max_ctx: int = 8192) -> list[int]:
    """Config 3's context lengths for a seed: U[1, max_ctx], one per request."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(1, max_ctx + 1, (batch,), generator=gen).tolist()


def workload_tensors(seed: int, device: torch.device, batch=64, num_heads=32, num_kv_heads=8,
                     head_dim=128, block_size=16, max_ctx=8192, dtype=torch.bfloat16) -> dict:
    """The config-3 step's inputs as plain tensors (no library types).

    Context lengths, the shuffled pool and the block tables come from CPU
    generators; K/V/Q and the new tokens from a generator on ``device``, so the
    GPU arm and the CPU reference arm (which draws on the GPU and copies to the
    host) see the same numbers.
    """
    lens = torch.tensor(workload_lens(seed, batch, max_ctx))
    gen = torch.Generator().manual_seed(seed + 7)
    need = (lens + block_size - 1) // block_size
    num_blocks = int(math.ceil(1.1 * int(need.sum())))
    perm = torch.randperm(num_blocks, generator=gen)
    width = int(need.max())
    tables = torch.zeros(batch, width, dtype=torch.int32)
    cursor = 0
    for b in range(batch):
        n = int(need[b])
        tables[b, :n] = perm[cursor:cursor + n].to(torch.int32)
        cursor += n
    shape = (1, num_blocks, block_size, num_kv_heads, head_dim)
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    k = torch.randn(shape, generator=dgen, device=device, dtype=dtype)
    v = torch.randn(shape, generator=dgen, device=device, dtype=dtype)
    query = torch.randn(batch, num_heads, head_dim, generator=dgen, device=device, dtype=dtype)
    new_k = torch.randn(batch, num_kv_heads, head_dim, generator=dgen, device=device, dtype=dtype)
    new_v = torch.randn(batch, num_kv_heads, head_dim, generator=dgen, device=device, dtype=dtype)
    pos = lens - 1  # the new token is the last position of each context
    slots = tables[torch.arange(batch), pos // block_size].long() * block_size + pos % block_size
    return dict(lens=lens.tolist(), tables=tables, num_blocks=num_blocks, k=k, v=v, query=query,
                new_k=new_k, new_v=new_v, slots=slots.to(torch.int32), block_size=block_size,
                num_heads=num_heads, num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=dtype)
