"""Prefix sharing on the host: refcounted blocks, the content index and the
runtime's lazy placement (CPU only; the GPU side is in test_gpu_llama.py)."""

import pytest

from inferkernellab_b200 import BlockAllocator, InferenceRuntime, PagedKVCache, TokenBudgetScheduler
from inferkernellab_b200.prefix_cache import PrefixCache, block_keys


def test_refcounted_free_returns_blocks_only_after_the_last_holder():
    alloc = BlockAllocator(6)
    a = alloc.allocate(3, owner=1)
    assert a == [0, 1, 2]
    alloc.share([1, 2])
    assert [alloc.ref_count(b) for b in a] == [1, 2, 2]
    alloc.free([1, 2], owner=7)  # shared: any holder may drop its reference
    assert alloc.num_used_blocks == 3 and alloc.ref_count(1) == 1
    with pytest.raises(ValueError, match="not owned"):
        alloc.free([1], owner=7)  # back to one holder: the owner check applies again
    alloc.free(a, owner=1)
    assert alloc.num_used_blocks == 0 and alloc.ref_count(1) == 0
    # LIFO reuse exactly as without sharing: last freed (2) comes out first.
    assert alloc.allocate(2) == [2, 1]
    with pytest.raises(ValueError, match="not allocated"):
        alloc.share([5])


def test_block_keys_chain_the_prefix():
    a = list(range(40))
    b = a[:35] + [99] * 10
    ka, kb = block_keys(a, 8), block_keys(b, 8)
    assert len(ka) == 5 and len(kb) == 5
    assert ka[:4] == kb[:4] and ka[4] != kb[4]
    # A different block 0 changes every later key even where the tokens match.
    c = [7] + a[1:]
    assert all(x != y for x, y in zip(block_keys(c, 8), ka))
    assert block_keys(a, 8, num_blocks=2) == ka[:2]


def test_prefix_cache_match_insert_evict():
    alloc = BlockAllocator(16)
    cache = PrefixCache(alloc, 8)
    tokens = list(range(40))
    table = alloc.allocate(5, owner=0)
    assert cache.match(tokens) == []
    assert cache.insert(tokens, table, 40) == 5
    assert all(alloc.ref_count(b) == 2 for b in table)
    # Longest cached prefix, capped so that the last token is computed again.
    got = cache.match(tokens)
    assert got == table[:4]
    assert alloc.ref_count(table[0]) == 3
    got2 = cache.match(tokens[:33] + [5, 5, 5])
    assert got2 == table[:4]
    alloc.free(got)
    alloc.free(got2)
    alloc.free(table, owner=0)  # the request is done; the cache still holds the blocks
    assert alloc.num_used_blocks == 5
    assert cache.evict(2) == 2 and alloc.num_used_blocks == 3
    cache.clear()
    assert alloc.num_used_blocks == 0 and len(cache) == 0


def _runtime(block_size=8, budget=48, num_blocks=64):
    cache = PagedKVCache(num_blocks, block_size, 1, 16, device="cpu")
    calls = []
    runtime = InferenceRuntime(
        cache, TokenBudgetScheduler(max_num_seqs=8, max_num_batched_tokens=budget),
        prefill_batch_fn=lambda reqs, s, e: calls.append(
            [(r.request_id, a, b, tuple(r.block_table)) for r, a, b in zip(reqs, s, e)]),
        decode_fn=lambda reqs: None, prefix_cache=PrefixCache(cache.allocator, block_size))
    return runtime, cache, calls


def test_runtime_places_requests_on_cached_prefixes():
    runtime, cache, calls = _runtime()
    a = list(range(40))
    b = a[:35] + list(range(100, 115))  # shares 4 full blocks with a
    c = list(a)                          # identical to a: shares 4 (the last token recomputed)
    runtime.submit(0, len(a), 1, token_ids=a)
    runtime.submit(1, len(b), 1, token_ids=b)
    runtime.submit(2, len(c), 1, token_ids=c)
    while runtime.scheduler.waiting or runtime.scheduler.running:
        runtime.step()
    flat = [x for batch in calls for x in batch]
    ranges = {rid: (s, e) for rid, s, e, _ in flat}
    tables = {rid: t for rid, _, _, t in flat}
    assert ranges == {0: (0, 40), 1: (32, 50), 2: (32, 40)}
    assert tables[1][:4] == tables[0][:4] and tables[2][:4] == tables[0][:4]
    assert tables[1][4] != tables[0][4]
    assert runtime.prefix_cached_tokens == 64
    # Finished requests dropped their references; only the index holds blocks.
    held = len(runtime.prefix_cache)
    assert cache.allocator.num_used_blocks == held
    runtime.prefix_cache.clear()
    assert cache.allocator.num_used_blocks == 0


def test_runtime_evicts_cached_blocks_when_the_pool_runs_short():
    runtime, cache, _ = _runtime(num_blocks=8, budget=64)
    first = list(range(40))
    runtime.submit(0, 40, 1, token_ids=first)
    while runtime.scheduler.waiting or runtime.scheduler.running:
        runtime.step()
    assert len(runtime.prefix_cache) == 5 and cache.allocator.num_free_blocks == 3
    other = list(range(500, 556))  # needs 7 blocks: 4 must come from evicted cache entries
    runtime.submit(1, 56, 1, token_ids=other)
    while runtime.scheduler.waiting or runtime.scheduler.running:
        runtime.step()
    assert len(runtime.prefix_cache) <= 7


def test_runtime_without_token_ids_is_unchanged():
    """No token ids: blocks at submit, exactly the reference behaviour."""
    runtime, cache, calls = _runtime()
    req = runtime.submit(0, 20, 1)
    assert req.block_table == [0, 1, 2]
    while runtime.scheduler.waiting or runtime.scheduler.running:
        runtime.step()
    assert calls[0][0][1:3] == (0, 20)
    assert len(runtime.prefix_cache) == 0
