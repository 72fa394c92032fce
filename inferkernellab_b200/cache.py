"""Paged KV cache storage and the physical-block allocator.

Host-side mirror of the reference's ``CacheLayout`` / ``BlockAllocator`` /
``PagedKVCache`` (reference ``src/inferkernellab/cache.py:8-200``): same
storage layout ``[layers, num_blocks, block_size, kv_heads, head_dim]``, same
deterministic allocation order (ids 0, 1, 2, ... then LIFO reuse), same
validation messages, so code written against the reference cache runs against
this one and vice versa.  The kernels of this package also accept the
reference's own ``PagedKVCache`` objects (they only read ``.k``, ``.v`` and
``.layout``).

Writes go through the sm_100a append kernel (``write``/``write_slots``); they
require the cache to live on a CUDA device.  ``read`` is an inspection helper
(a torch gather) and is not used by any kernel path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class CacheLayout:
    num_layers: int
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int


class BlockAllocator:
    """Deterministic physical-block allocator with owner tracking and sharing.

    ``allocate`` hands out the lowest never-used ids first (0, 1, 2, ...) and
    reuses freed ids last-freed-first, matching reference ``cache.py:17-64``;
    ``free`` validates the whole request before releasing anything.

    Blocks carry a reference count (prefix sharing, ``prefix_cache.py``):
    ``share`` adds a holder to allocated blocks and ``free`` drops one; a block
    returns to the free stack when its last holder frees it.  A block with a
    single holder behaves exactly as in the reference (same order, same owner
    checks); the owner check is skipped for blocks that are shared.
    """

    def __init__(self, num_blocks: int):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self._capacity = num_blocks
        # Stack of free ids; the top (end) is handed out next.
        self._stack = list(range(num_blocks - 1, -1, -1))
        self._in_use: set[int] = set()
        self._owner_of: dict[int, int] = {}
        self._refs: dict[int, int] = {}

    @property
    def num_free_blocks(self) -> int:
        return len(self._stack)

    @property
    def num_used_blocks(self) -> int:
        return len(self._in_use)

    def allocate(self, count: int, owner: int | None = None) -> list[int]:
        if count < 0:
            raise ValueError("count must be non-negative")
        if count > len(self._stack):
            raise RuntimeError(f"out of KV blocks: requested={count}, free={len(self._stack)}")
        taken = [self._stack.pop() for _ in range(count)]
        self._in_use.update(taken)
        self._refs.update((block, 1) for block in taken)
        if owner is not None:
            self._owner_of.update((block, owner) for block in taken)
        return taken

    def free(self, block_ids, owner: int | None = None) -> None:
        ids = tuple(block_ids)
        if len(ids) != len(set(ids)):
            raise ValueError("block_ids must not contain duplicates")
        for block in ids:  # validate everything first: the free is all-or-nothing
            if not isinstance(block, int) or not 0 <= block < self._capacity:
                raise ValueError(f"invalid block id: {block}")
            if block not in self._in_use:
                raise ValueError(f"block {block} is not allocated")
            if (owner is not None and self._refs.get(block, 1) == 1
                    and self._owner_of.get(block) != owner):
                raise ValueError(f"block {block} is not owned by request {owner}")
        for block in ids:
            refs = self._refs.get(block, 1) - 1
            if refs > 0:
                self._refs[block] = refs
                continue
            self._refs.pop(block, None)
            self._in_use.discard(block)
            self._owner_of.pop(block, None)
            self._stack.append(block)

    def share(self, block_ids) -> None:
        """Add one holder to each allocated block of ``block_ids``."""
        ids = tuple(block_ids)
        for block in ids:
            if not isinstance(block, int) or block not in self._in_use:
                raise ValueError(f"block {block} is not allocated")
        for block in ids:
            self._refs[block] = self._refs.get(block, 1) + 1

    def ref_count(self, block_id: int) -> int:
        """Holders of ``block_id`` (0 when it is free)."""
        return self._refs.get(block_id, 0) if block_id in self._in_use else 0

    def owner(self, block_id: int) -> int | None:
        return self._owner_of.get(block_id)


class PagedKVCache:
    """K/V storage in physical blocks plus a block allocator (reference ``cache.py:67-200``)."""

    def __init__(self, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int, *,
                 num_layers: int = 1, dtype: torch.dtype = torch.float16,
                 device: torch.device | str = "cpu"):
        if min(num_layers, num_blocks, block_size, num_kv_heads, head_dim) <= 0:
            raise ValueError("cache dimensions must be positive")
        self.layout = CacheLayout(num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.k = torch.empty(shape, dtype=dtype, device=torch.device(device))
        self.v = torch.empty_like(self.k)
        self.device = self.k.device
        self.allocator = BlockAllocator(num_blocks)

    @property
    def dtype(self) -> torch.dtype:
        return self.k.dtype

    @property
    def numel_bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()

    def allocate_request(self, request_id: int, num_tokens: int) -> list[int]:
        if num_tokens <= 0:
            raise ValueError("num_tokens must be positive")
        blocks_needed = -(-num_tokens // self.layout.block_size)
        return self.allocator.allocate(blocks_needed, owner=request_id)

    def release_request(self, block_table, request_id: int | None = None) -> None:
        self.allocator.free(block_table, owner=request_id)

    def slot_mapping(self, block_table, start: int, length: int) -> torch.Tensor:
        """int64 physical slots of logical tokens ``start .. start+length-1``.

        Same checks, messages and formula as reference ``cache.py:113-129``;
        the slots are computed on the host (where the table lives) and copied
        once to the cache device.  The device-side builder for whole batches is
        ``inferkernellab_b200.ops.build_slot_mapping``.
        """
        if start < 0 or length < 0:
            raise ValueError("start and length must be non-negative")
        bs = self.layout.block_size
        if isinstance(block_table, torch.Tensor):
            if block_table.ndim != 1:
                raise ValueError("block_table must be one-dimensional")
            table = [int(b) for b in block_table.tolist()]
        else:
            if any(not isinstance(b, int) or not 0 <= b < self.layout.num_blocks
                   for b in block_table):
                raise ValueError("block_table contains an invalid physical block id")
            table = list(block_table)
        if length and (start + length - 1) // bs >= len(table):
            raise ValueError("block_table is shorter than the requested range")
        slots = [table[p // bs] * bs + p % bs for p in range(start, start + length)]
        return torch.tensor(slots, dtype=torch.long).to(self.device)

    def write(self, layer: int, block_table, start: int, key: torch.Tensor,
              value: torch.Tensor) -> None:
        """Write ``[T, kv_heads, head_dim]`` into logical positions ``start ..``."""
        if key.shape != value.shape or key.ndim != 3:
            raise ValueError("key/value must have the same [T, H, D] shape")
        if tuple(key.shape[1:]) != (self.layout.num_kv_heads, self.layout.head_dim):
            raise ValueError("key/value shape does not match cache layout")
        slots = self.slot_mapping(block_table, start, key.shape[0])
        if not 0 <= layer < self.layout.num_layers:
            raise IndexError("layer is out of range")
        from .ops import append_kv  # local import: ops imports this module

        append_kv(key.to(self.device), value.to(self.device), self, slots, layer=layer)

    def write_slots(self, layer: int, slots: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                    *, validate_slots: bool = True) -> None:
        """Write flattened tokens to physical ``slots`` (reference ``cache.py:156-189``)."""
        if key.shape != value.shape or key.ndim != 3:
            raise ValueError("key/value must have the same [T, H, D] shape")
        if slots.ndim != 1 or slots.numel() != key.shape[0]:
            raise ValueError("slots must have one entry per key/value token")
        if tuple(key.shape[1:]) != (self.layout.num_kv_heads, self.layout.head_dim):
            raise ValueError("key/value shape does not match cache layout")
        if not 0 <= layer < self.layout.num_layers:
            raise IndexError("layer is out of range")
        slots = slots.to(self.device)
        if validate_slots and slots.numel():
            limit = self.layout.num_blocks * self.layout.block_size
            if bool((slots < 0).any()) or bool((slots >= limit).any()):
                raise ValueError("slots contain an invalid physical cache position")
        from .ops import append_kv

        append_kv(key.to(self.device), value.to(self.device), self, slots, layer=layer)

    def read(self, layer: int, block_table, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        """First ``length`` logical tokens in order (inspection helper, torch gather)."""
        if length < 0:
            raise ValueError("length must be non-negative")
        slots = self.slot_mapping(block_table, 0, length)
        if not 0 <= layer < self.layout.num_layers:
            raise IndexError("layer is out of range")
        bs = self.layout.block_size
        return self.k[layer, slots // bs, slots % bs], self.v[layer, slots // bs, slots % bs]
