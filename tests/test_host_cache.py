"""Host logic of the cache and allocator (mirrors reference tests/test_cache.py)."""

import pytest
import torch

from inferkernellab_b200 import BlockAllocator, PagedKVCache


def test_slot_mapping_crosses_physical_blocks():
    cache = PagedKVCache(8, 4, 2, 16, dtype=torch.float16)
    assert cache.slot_mapping([6, 2, 5], 2, 6).tolist() == [26, 27, 8, 9, 10, 11]
    assert cache.slot_mapping([6, 2, 5], 2, 6).dtype == torch.long


def test_slot_mapping_tensor_table_and_empty_range():
    cache = PagedKVCache(8, 4, 2, 16, dtype=torch.float16)
    assert cache.slot_mapping(torch.tensor([6, 2, 5]), 0, 3).tolist() == [24, 25, 26]
    assert cache.slot_mapping([6], 0, 0).tolist() == []
    with pytest.raises(ValueError, match="one-dimensional"):
        cache.slot_mapping(torch.tensor([[6, 2]]), 0, 1)


def test_slot_mapping_rejects_invalid_physical_blocks():
    cache = PagedKVCache(4, 4, 1, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="invalid physical block"):
        cache.slot_mapping([-1], 0, 1)
    with pytest.raises(ValueError, match="shorter"):
        cache.slot_mapping([2], 4, 1)
    with pytest.raises(ValueError, match="non-negative"):
        cache.slot_mapping([2], -1, 1)


def test_allocator_order_is_deterministic_and_lifo():
    allocator = BlockAllocator(6)
    assert allocator.allocate(3, owner=1) == [0, 1, 2]
    assert allocator.allocate(1, owner=2) == [3]
    allocator.free([1, 2], owner=1)
    assert allocator.allocate(2, owner=3) == [2, 1]
    with pytest.raises(RuntimeError, match="out of KV blocks"):
        allocator.allocate(4)
    with pytest.raises(ValueError, match="non-negative"):
        allocator.allocate(-1)


def test_allocator_releases_blocks():
    cache = PagedKVCache(4, 4, 1, 16, dtype=torch.float16)
    table = cache.allocate_request(7, 5)
    assert cache.allocator.num_free_blocks == 2
    cache.release_request(table)
    assert cache.allocator.num_free_blocks == 4
    with pytest.raises(ValueError, match="positive"):
        cache.allocate_request(1, 0)


def test_allocator_rejects_invalid_free_atomically():
    allocator = BlockAllocator(4)
    blocks = allocator.allocate(2, owner=7)
    with pytest.raises(ValueError, match="not allocated"):
        allocator.free([blocks[0], 3])
    with pytest.raises(ValueError, match="invalid block id"):
        allocator.free([9])
    assert allocator.num_used_blocks == 2 and allocator.num_free_blocks == 2
    with pytest.raises(ValueError, match="duplicates"):
        allocator.free([blocks[0], blocks[0]])
    with pytest.raises(ValueError, match="not owned"):
        allocator.free(blocks, owner=8)
    assert allocator.num_used_blocks == 2
    assert allocator.owner(blocks[0]) == 7
    allocator.free(blocks, owner=7)
    assert allocator.num_used_blocks == 0 and allocator.num_free_blocks == 4


def test_cache_validation_and_layout():
    with pytest.raises(ValueError, match="positive"):
        PagedKVCache(0, 4, 1, 16)
    cache = PagedKVCache(5, 8, 2, 32, num_layers=3, dtype=torch.bfloat16)
    assert tuple(cache.k.shape) == (3, 5, 8, 2, 32)
    assert cache.numel_bytes == 2 * 3 * 5 * 8 * 2 * 32 * 2
    assert cache.dtype == torch.bfloat16


def test_ragged_list_tables_pad_with_block_zero():
    # The reference's paged_reference backend hands the operators one Python
    # list per request; rows past a request's context are never read.
    from inferkernellab_b200.ops import _as_table_tensor

    cpu = torch.device("cpu")
    t = _as_table_tensor([[3, 1, 4], [1], (5, 9)], cpu)
    assert t.dtype == torch.int32 and t.tolist() == [[3, 1, 4], [1, 0, 0], [5, 9, 0]]
    assert _as_table_tensor([[2, 7], [1, 8]], cpu).tolist() == [[2, 7], [1, 8]]
    dev = torch.zeros(2, 3, dtype=torch.int64)
    assert _as_table_tensor(dev, cpu) is dev
