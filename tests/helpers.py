"""Seeded input builders shared by the tests (torch tensors + numpy oracle views)."""

from __future__ import annotations

import numpy as np
import torch

# Tolerances of the CUDA path against the float32 oracle.
TOL = {torch.float16: dict(atol=2e-3, rtol=1e-2), torch.bfloat16: dict(atol=1e-2, rtol=2e-2)}
KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}


def to_np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy in the oracle's storage convention (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def from_np(a: np.ndarray, kind: str, device="cpu") -> torch.Tensor:
    if kind == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


class DecodeCase:
    """A paged cache filled with N(0,1) data, shuffled block tables and a query."""

    def __init__(self, *, batch, num_heads, num_kv_heads, head_dim, block_size, lens, dtype,
                 seed=0, num_blocks=None, layers=1, layer=0, table_dtype=torch.int32,
                 width=None, nan_fill=False, device="cuda"):
        from inferkernellab_b200 import PagedKVCache

        gen = torch.Generator().manual_seed(seed)
        need = [-(-n // block_size) for n in lens]
        total = sum(need)
        num_blocks = num_blocks or max(1, int(total * 1.1) + 1)
        self.cache = PagedKVCache(num_blocks, block_size, num_kv_heads, head_dim,
                                  num_layers=layers, dtype=dtype, device=device)
        k = torch.randn(self.cache.k.shape, generator=gen).to(dtype)
        v = torch.randn(self.cache.v.shape, generator=gen).to(dtype)
        if nan_fill:
            k.fill_(float("nan"))
            v.fill_(float("nan"))
        perm = torch.randperm(num_blocks, generator=gen).tolist()
        width = width or max(need)
        rows, cursor = [], 0
        for n in need:
            row = perm[cursor:cursor + n]
            cursor += n
            rows.append(row + [0] * (width - len(row)))
        if nan_fill:
            # Only the tokens inside each context are real values.
            for b, n in enumerate(lens):
                for p in range(n):
                    blk, off = rows[b][p // block_size], p % block_size
                    k[layer, blk, off] = torch.randn(num_kv_heads, head_dim, generator=gen).to(dtype)
                    v[layer, blk, off] = torch.randn(num_kv_heads, head_dim, generator=gen).to(dtype)
        self.cache.k.copy_(k)
        self.cache.v.copy_(v)
        self.tables_list = rows
        self.lens_list = list(lens)
        self.tables = torch.tensor(rows, dtype=table_dtype, device=device)
        self.lens = torch.tensor(lens, dtype=table_dtype, device=device)
        self.query = torch.randn(batch, num_heads, head_dim, generator=gen).to(dtype).to(device)
        self.dtype = dtype
        self.layer = layer
        self.kind = KIND[dtype]

    def oracle(self, scale=None):
        from oracle import paged_decode_attention

        return paged_decode_attention(to_np(self.query), to_np(self.cache.k), to_np(self.cache.v),
                                      self.kind, self.tables_list, self.lens_list, scale=scale,
                                      layer=self.layer)


def assert_close(actual: torch.Tensor, expected: np.ndarray, dtype, what=""):
    got = actual.detach().float().cpu().numpy()
    tol = TOL[dtype]
    ok = np.allclose(got, expected, atol=tol["atol"], rtol=tol["rtol"])
    if not ok:
        diff = np.abs(got - expected)
        bad = ~np.isclose(got, expected, atol=tol["atol"], rtol=tol["rtol"])
        idx = np.argwhere(bad)[:5]
        raise AssertionError(
            f"{what}: max abs err {np.nanmax(diff):.3e}, {bad.sum()} / {bad.size} outside "
            f"atol={tol['atol']} rtol={tol['rtol']}; first bad {idx.tolist()} "
            f"got {got[tuple(idx[0])] if len(idx) else None} want {expected[tuple(idx[0])] if len(idx) else None}")
