"""Parity of the append, prefill and metadata kernels with the oracle.

Append and slot mapping are bit-exact (torch.equal / array_equal).  Prefill uses
the tolerances of tests/helpers.TOL against the float32 restatement of the
reference's paged_prefill_attention_sdpa (attention.py:230-321).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import (
    PagedKVCache,
    append_kv,
    build_slot_mapping,
    check_device_errors,
    paged_prefill_attention,
    paged_prefill_attention_varlen,
)
from tests.helpers import KIND, assert_close, from_np, to_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------------ append

def test_append_matches_reference_golden_bit_exact():
    d = np.load(GOLDEN / "append.npz")
    cache = PagedKVCache(8, 8, 2, 16, num_layers=2, dtype=torch.float16, device="cuda")
    cache.k.zero_()
    cache.v.zero_()
    append_kv(from_np(d["key"], "f16", "cuda"), from_np(d["value"], "f16", "cuda"), cache,
              torch.tensor(d["slots"], device="cuda"), layer=int(d["layer"]))
    assert np.array_equal(to_np(cache.k).view(np.uint16), d["k_after"].view(np.uint16))
    assert np.array_equal(to_np(cache.v).view(np.uint16), d["v_after"].view(np.uint16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("dim,bs,hkv", [(64, 16, 8), (128, 16, 8), (16, 8, 2), (32, 4, 1)])
def test_append_bit_exact_against_oracle(dtype, slot_dtype, dim, bs, hkv):
    gen = torch.Generator().manual_seed(dim * 7 + bs)
    nb, layers, tokens = 40, 2, 77
    cache = PagedKVCache(nb, bs, hkv, dim, num_layers=layers, dtype=dtype, device="cuda")
    base_k = torch.randn(cache.k.shape, generator=gen).to(dtype)
    base_v = torch.randn(cache.v.shape, generator=gen).to(dtype)
    cache.k.copy_(base_k)
    cache.v.copy_(base_v)
    slots = torch.randperm(nb * bs, generator=gen)[:tokens]
    key = torch.randn(tokens, hkv, dim, generator=gen).to(dtype)
    value = torch.randn(tokens, hkv, dim, generator=gen).to(dtype)
    append_kv(key.cuda(), value.cuda(), cache, slots.to(slot_dtype).cuda(), layer=1)
    k_np, v_np = to_np(base_k), to_np(base_v)
    oracle.write_slots(k_np, v_np, 1, slots.numpy(), to_np(key), to_np(value))
    assert np.array_equal(to_np(cache.k), k_np)
    assert np.array_equal(to_np(cache.v), v_np)


def test_append_strided_source_negative_slots_and_bad_slots():
    gen = torch.Generator().manual_seed(1)
    cache = PagedKVCache(4, 8, 2, 64, dtype=torch.bfloat16, device="cuda")
    cache.k.zero_()
    cache.v.zero_()
    # [T, Hkv, D] views with a token stride of 3 heads (non-contiguous, still 16B aligned).
    big = torch.randn(6, 3, 64, generator=gen).to(torch.bfloat16).cuda()
    key, value = big[:, :2], big[:, 1:]
    slots = torch.tensor([0, -1, 5, 31, 32, 9], dtype=torch.int64, device="cuda")
    append_kv(key, value, cache, slots)
    k_np = np.zeros(to_np(cache.k).shape, np.uint16)
    v_np = np.zeros_like(k_np)
    keep = [0, 2, 3, 5]
    oracle.write_slots(k_np, v_np, 0, slots.cpu().numpy()[keep], to_np(key)[keep], to_np(value)[keep])
    assert np.array_equal(to_np(cache.k), k_np)
    assert np.array_equal(to_np(cache.v), v_np)
    assert check_device_errors() & 4  # slot 32 is past the pool: DEVERR_BAD_SLOT


def test_cache_write_and_read_preserve_logical_order():
    cache = PagedKVCache(8, 4, 2, 16, dtype=torch.float16, device="cuda")
    table = [5, 1]
    key = torch.arange(2 * 2 * 16, dtype=torch.float16).view(2, 2, 16).cuda()
    value = key + 100
    cache.write(0, table, 2, key, value)
    read_key, read_value = cache.read(0, table, 4)
    assert torch.equal(read_key[2:], key) and torch.equal(read_value[2:], value)
    slots = torch.cat((cache.slot_mapping([6, 2, 5], 0, 2), cache.slot_mapping([6, 2, 5], 4, 2)))
    key2 = torch.randn(4, 2, 16, dtype=torch.float16, device="cuda")
    cache.write_slots(0, slots, key2, key2 + 1)
    k, v = cache.read(0, [6, 2, 5], 6)
    assert torch.equal(k[[0, 1, 4, 5]], key2) and torch.equal(v[[0, 1, 4, 5]], key2 + 1)
    with pytest.raises(ValueError, match="invalid physical cache position"):
        cache.write_slots(0, torch.tensor([32], device="cuda"), key2[:1], key2[:1])


# ----------------------------------------------------------------- prefill

@pytest.mark.parametrize("path", sorted(GOLDEN.glob("prefill_*.npz")), ids=lambda p: p.stem)
def test_prefill_matches_reference_golden(path):
    d = np.load(path)
    kind = str(d["kind"])
    dtype = torch.bfloat16 if kind == "bf16" else torch.float16
    k = from_np(d["k"], kind, "cuda")
    layers, nb, bs, hkv, dim = k.shape
    cache = PagedKVCache(nb, bs, hkv, dim, num_layers=layers, dtype=dtype, device="cuda")
    cache.k.copy_(k)
    cache.v.copy_(from_np(d["v"], kind, "cuda"))
    out = paged_prefill_attention(from_np(d["query"], kind, "cuda"), cache,
                                  d["block_tables"].tolist(), d["query_starts"].tolist(),
                                  d["context_lens"].tolist())
    assert_close(out, d["out_f32"], dtype, path.stem)  # padded rows included


def _prefill_case(dtype, hq, hkv, dim, bs, starts, ends, seed, nan_fill=False):
    gen = torch.Generator().manual_seed(seed)
    need = [-(-e // bs) for e in ends]
    nb = sum(need) + 3
    cache = PagedKVCache(nb, bs, hkv, dim, dtype=dtype, device="cuda")
    fill = float("nan") if nan_fill else None
    k = torch.randn(cache.k.shape, generator=gen).to(dtype)
    v = torch.randn(cache.v.shape, generator=gen).to(dtype)
    if fill is not None:
        k.fill_(fill)
        v.fill_(fill)
    perm = torch.randperm(nb, generator=gen).tolist()
    width = max(need)
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [0] * (width - n))
        cur += n
    cache.k.copy_(k)
    cache.v.copy_(v)
    # Append the real tokens [0, end) through the kernel under test's sibling.
    for b, e in enumerate(ends):
        kk = torch.randn(e, hkv, dim, generator=gen).to(dtype).cuda()
        vv = torch.randn(e, hkv, dim, generator=gen).to(dtype).cuda()
        cache.write(0, tables[b], 0, kk, vv)
    width_q = max(e - s for s, e in zip(starts, ends))
    query = torch.randn(len(ends), hq, width_q, dim, generator=gen).to(dtype).cuda()
    return cache, tables, query


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("cfg", [
    (32, 8, 128, 16, [0, 0, 100], [300, 17, 229]),   # config-4 like: D128 GQA, chunk continuation
    (8, 8, 64, 16, [0, 5], [64, 70]),                # MHA, exact tile boundary
    (32, 1, 64, 16, [0], [150]),                     # MQA
    (4, 2, 16, 4, [0, 2], [5, 7]),                   # the reference's ragged test geometry
    (6, 3, 32, 8, [10, 0], [43, 9]),
    (8, 2, 128, 256, [0, 200], [513, 300]),          # big pages
])
def test_prefill_padded_matches_oracle(cfg, dtype):
    hq, hkv, dim, bs, starts, ends = cfg
    cache, tables, query = _prefill_case(dtype, hq, hkv, dim, bs, starts, ends, seed=len(ends) + dim)
    out = paged_prefill_attention(query, cache, tables, starts, ends)
    want = oracle.paged_prefill_attention(to_np(query), to_np(cache.k), to_np(cache.v), KIND[dtype],
                                          tables, starts, ends)
    assert_close(out, want, dtype, str(cfg))


def test_prefill_varlen_matches_padded_and_skips_nan_slots():
    dtype = torch.bfloat16
    starts, ends = [0, 33, 7], [97, 50, 8]
    cache, tables, query = _prefill_case(dtype, 16, 4, 64, 16, starts, ends, seed=77, nan_fill=True)
    padded = paged_prefill_attention(query, cache, tables, starts, ends)
    lens = [e - s for s, e in zip(starts, ends)]
    packed = torch.cat([query[b, :, :n].transpose(0, 1) for b, n in enumerate(lens)]).contiguous()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    out = paged_prefill_attention_varlen(
        packed, cache, torch.tensor(tables, dtype=torch.int32, device="cuda"), cu,
        torch.tensor(starts, dtype=torch.int32, device="cuda"),
        torch.tensor(ends, dtype=torch.int32, device="cuda"))
    ref = torch.cat([padded[b, :, :n].transpose(0, 1) for b, n in enumerate(lens)])
    assert torch.isfinite(out).all()
    assert torch.equal(out, ref)  # same kernel math, different addressing
    want = oracle.paged_prefill_attention(to_np(query), to_np(cache.k), to_np(cache.v), "bf16",
                                          tables, starts, ends)
    assert_close(padded, want, dtype, "varlen nan")


@pytest.mark.parametrize("kernel", ["tcgen05", "mma_sync"])
def test_prefill_padded_without_validation_never_synchronises(kernel):
    """validate_inputs=False with device ranges: no host synchronisation (torch's
    sync debug mode raises on one) and the same output as the validating call."""
    dtype = torch.bfloat16
    starts, ends = [0, 33, 7], [97, 50, 8]
    cache, tables, query = _prefill_case(dtype, 16, 4, 64, 16, starts, ends, seed=5)
    want = paged_prefill_attention(query, cache, tables, starts, ends, kernel=kernel)
    tables_d = torch.tensor(tables, dtype=torch.int32, device="cuda")
    starts_d = torch.tensor(starts, dtype=torch.int32, device="cuda")
    ends_d = torch.tensor(ends, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = paged_prefill_attention(query, cache, tables_d, starts_d, ends_d, kernel=kernel,
                                      validate_inputs=False)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    assert torch.equal(out, want)


def test_prefill_rejects_bad_ranges():
    cache = PagedKVCache(8, 4, 2, 16, dtype=torch.float16, device="cuda")
    query = torch.randn(1, 4, 4, 16, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="non-empty"):
        paged_prefill_attention(query, cache, [[0, 1]], [3], [3])
    with pytest.raises(ValueError, match="width"):
        paged_prefill_attention(query, cache, [[0, 1]], [0], [6])
    with pytest.raises(ValueError, match="capacity"):
        paged_prefill_attention(query, cache, [[0]], [2], [6])
    with pytest.raises(IndexError):
        paged_prefill_attention(query, cache, [[0, 1]], [0], [3], layer=2)


# ---------------------------------------------------------------- metadata

@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_build_slot_mapping_matches_host_slot_mapping(index_dtype):
    gen = torch.Generator().manual_seed(11)
    bs, nb = 16, 300
    starts = [0, 37, 500, 3, 0]
    ends = [19, 300, 512, 4, 1]
    width = max(-(-e // bs) for e in ends)
    perm = torch.randperm(nb, generator=gen).tolist()
    tables = [perm[i * width:(i + 1) * width] for i in range(len(ends))]
    want = np.concatenate([oracle.slot_mapping(t, s, e - s, bs, nb)
                           for t, s, e in zip(tables, starts, ends)])
    total = int(sum(e - s for s, e in zip(starts, ends)))
    for slots_dtype in (torch.int32, torch.int64):
        slots, cu = build_slot_mapping(
            torch.tensor(tables, dtype=index_dtype, device="cuda"),
            torch.tensor(starts, dtype=index_dtype, device="cuda"),
            torch.tensor(ends, dtype=index_dtype, device="cuda"),
            block_size=bs, num_blocks=nb, total_tokens=total, slots_dtype=slots_dtype)
        assert slots.dtype == slots_dtype
        assert np.array_equal(slots.cpu().numpy().astype(np.int64), want)
        assert cu.cpu().tolist() == [0] + list(np.cumsum([e - s for s, e in zip(starts, ends)]))
    assert check_device_errors() == 0


def test_build_slot_mapping_flags_out_of_table_positions():
    tables = torch.tensor([[3, 1], [2, 9]], dtype=torch.int32, device="cuda")
    slots, _ = build_slot_mapping(tables, torch.tensor([0, 0], device="cuda"),
                                  torch.tensor([3, 6], device="cuda"), block_size=2,
                                  num_blocks=5, total_tokens=9)
    # request 1: block 9 is outside the pool, position 4-5 past the table.
    assert slots.cpu().tolist() == [6, 7, 2, 4, 5, -1, -1, -1, -1]
    assert check_device_errors() & 8
