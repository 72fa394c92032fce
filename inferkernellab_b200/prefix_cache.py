"""Prefix sharing over the paged KV cache: refcounted full blocks keyed by content.

A block table already lets several requests point at one physical block; what a
serving loop needs on top is (1) reference counts, so a block shared by several
requests is freed only by its last holder (``BlockAllocator.share``/``free``),
and (2) an index from *prompt content* to the physical blocks that already hold
its K/V.  ``PrefixCache`` is that index.

* A key is a chained 128-bit BLAKE2b digest of a full block of token ids and
  every block before it (block ``i``'s key covers tokens ``0 ..
  (i+1)*block_size - 1``), so equal keys mean equal token prefixes at equal
  positions -- hence identical K/V for a deterministic model.  Only full
  blocks are shared; the block a request is still writing into is its own.
* ``match(tokens)`` returns the physical blocks of the longest cached prefix,
  capped so that at least the last prompt token is computed again (the model
  needs that token's logits).  The caller's block table starts with them and
  its prefill starts after them.
* ``insert(tokens, block_table, num_tokens)`` registers the full blocks of a
  request whose first ``num_tokens`` tokens are in the cache.  The index holds
  one reference per cached block, so cached K/V survives the request.
* ``evict(count)`` releases least-recently-used entries that nobody else holds
  (reference count 1), so the allocator can reuse them; ``InferenceRuntime``
  calls it when an allocation would fail.

This is the reference's "prefix sharing / refcounted blocks on top of
BlockAllocator" item (``docs/design.md:18`` of the reference project); the
reference itself has no implementation, so its behaviour is pinned against the
unshared path instead (same tokens, same logits).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict
from collections.abc import Sequence


def block_keys(tokens: Sequence[int], block_size: int,
               num_blocks: int | None = None) -> list[bytes]:
    """Chained content keys of the first ``num_blocks`` full blocks of ``tokens``:
    ``key_i = BLAKE2b-128(key_{i-1} || token ids of block i as int64)``."""
    full = len(tokens) // block_size
    if num_blocks is not None:
        full = min(full, num_blocks)
    keys, parent = [], b""
    for i in range(full):
        block = tokens[i * block_size:(i + 1) * block_size]
        data = b"".join(int(t).to_bytes(8, "little", signed=True) for t in block)
        parent = hashlib.blake2b(parent + data, digest_size=16).digest()
        keys.append(parent)
    return keys


class PrefixCache:
    def __init__(self, allocator, block_size: int):
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.allocator = allocator
        self.block_size = block_size
        self._blocks: OrderedDict[bytes, int] = OrderedDict()  # key -> physical block, LRU order
        self.hits = 0       # blocks served from the cache
        self.queries = 0    # full prompt blocks looked up

    def __len__(self) -> int:
        return len(self._blocks)

    def lookup(self, tokens: Sequence[int]) -> list[int]:
        """Physical blocks of the longest cached prefix of ``tokens``, capped so that
        at least the last token is computed again; no reference is taken."""
        usable = (len(tokens) - 1) // self.block_size
        found = []
        for key in block_keys(tokens, self.block_size, usable):
            block = self._blocks.get(key)
            if block is None:
                break
            found.append(block)
        return found

    def match(self, tokens: Sequence[int]) -> list[int]:
        """``lookup`` that takes the blocks: each gets one more holder (the caller
        owns that reference and frees it like its own) and becomes most recent."""
        usable = (len(tokens) - 1) // self.block_size
        found = []
        for key in block_keys(tokens, self.block_size, usable):
            block = self._blocks.get(key)
            if block is None:
                break
            self._blocks.move_to_end(key)
            found.append(block)
        self.queries += usable
        self.hits += len(found)
        if found:
            self.allocator.share(found)
        return found

    def insert(self, tokens: Sequence[int], block_table: Sequence[int], num_tokens: int) -> int:
        """Index the full blocks among the first ``num_tokens`` tokens; returns how many
        new blocks the cache now holds."""
        full = min(num_tokens, len(tokens)) // self.block_size
        added = 0
        for i, key in enumerate(block_keys(tokens, self.block_size, full)):
            if i >= len(block_table):
                break
            if key in self._blocks:
                self._blocks.move_to_end(key)
                continue
            block = int(block_table[i])
            self.allocator.share([block])
            self._blocks[key] = block
            added += 1
        return added

    def evict(self, count: int) -> int:
        """Release up to ``count`` least-recently-used blocks held only by the cache."""
        freed = 0
        for key in list(self._blocks):
            if freed >= count:
                break
            block = self._blocks[key]
            if self.allocator.ref_count(block) == 1:
                del self._blocks[key]
                self.allocator.free([block])
                freed += 1
        return freed

    def clear(self) -> None:
        """Drop every entry (blocks still held by requests stay allocated)."""
        for block in self._blocks.values():
            self.allocator.free([block])
        self._blocks.clear()
