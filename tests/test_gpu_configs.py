"""Parity at the BASELINE.json configurations the benchmarks run, at full size.

* config 3 -- the exact step ``bench.py`` times (seed 0, 64 requests, ctx
  U[1, 8192], Hq32/Hkv8, D128, BS16, bf16, pool 1.1x shuffled; one
  ``paged_decode_attention_append`` launch with the plain append): cache bits
  against the oracle's ``write_slots`` and the output against the oracle's
  ``paged_decode_attention`` (reference ``cache.py:156-189``,
  ``attention.py:134-175``);
* config 2 -- the whole 36-shape grid B{1,4,16} x ctx{128,512} x Hkv{32,8,1} x
  fp16/bf16 (Hq32, D64, BS16, shuffled pool): append one token per request
  through its slot, then attend over ctx + 1, both as two launches
  (``append_kv`` + ``paged_decode_attention``) and fused (reference
  ``scripts/run_decode_sweep.py:261-369`` sweeps the same grid);
* config 4 -- 24 seeded prompts U[17, 512] packed by ``TokenBudgetScheduler``
  under a 2048-token budget (``benchmark.config4_plan``), each budget batch run
  as ``build_slot_mapping`` -> (``rope_append_kv`` | ``append_kv``) ->
  ``paged_prefill_attention_varlen`` on both prefill kernels, over a cache
  poisoned with NaN: slots, rotated query and cache bits exact, attention
  within the bf16 bar of the oracle.

Tolerances are the north-star bars in ``tests/helpers.TOL`` (fp16 atol 2e-3 /
rtol 1e-2, bf16 atol 1e-2 / rtol 2e-2) against the float32 oracle.
"""

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import (
    PagedKVCache,
    append_kv,
    build_slot_mapping,
    check_device_errors,
    paged_decode_attention,
    paged_decode_attention_append,
    paged_prefill_attention_varlen,
    rope_append_kv,
)
from inferkernellab_b200.benchmark import config4_plan
from tests.helpers import KIND, DecodeCase, assert_close, to_np

pytestmark = pytest.mark.gpu


def _oracle_decode(query, k, v, kind, tables, lens):
    """The oracle's paged decode, one request per worker thread."""
    def one(b):
        return oracle.paged_decode_attention(query[b:b + 1], k, v, kind, [tables[b]], [lens[b]])[0]

    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as pool:
        return np.stack(list(pool.map(one, range(len(lens)))))


# ------------------------------------------------------------------ config 3

def test_config3_bench_step_matches_oracle():
    import bench

    check_device_errors()
    wl = bench.Workload(seed=0, device=torch.device("cuda", torch.cuda.current_device()))
    assert wl.batch == 64 and sum(wl.lens_list) == 263090  # the bench line's sum_ctx_rank0
    k_want, v_want = to_np(wl.cache.k), to_np(wl.cache.v)
    oracle.write_slots(k_want, v_want, 0, wl.slots_host.tolist(), to_np(wl.new_k),
                       to_np(wl.new_v))
    wl.step()
    torch.cuda.synchronize()
    assert np.array_equal(to_np(wl.cache.k), k_want), "K cache differs from the oracle append"
    assert np.array_equal(to_np(wl.cache.v), v_want), "V cache differs from the oracle append"
    bs = wl.block_size
    tables = [wl.tables_host[b, :-(-n // bs)].tolist() for b, n in enumerate(wl.lens_list)]
    want = _oracle_decode(to_np(wl.query), k_want, v_want, "bf16", tables, wl.lens_list)
    assert_close(wl.out, want, torch.bfloat16, "config-3 bench step")
    first = wl.out.clone()
    wl.step()  # idempotent: the same slots are rewritten with the same values
    assert torch.equal(wl.out, first)
    assert check_device_errors() == 0


# ------------------------------------------------------------------ config 2

CONFIG2 = [(b, ctx, hkv, dt) for dt in (torch.float16, torch.bfloat16) for b in (1, 4, 16)
           for ctx in (128, 512) for hkv in (32, 8, 1)]


@pytest.mark.parametrize("fused", [False, True], ids=["two_launches", "fused"])
@pytest.mark.parametrize("batch,ctx,hkv,dtype", CONFIG2,
                         ids=[f"B{b}-ctx{c}-Hkv{h}-{KIND[d]}" for b, c, h, d in CONFIG2])
def test_config2_append_then_decode_matches_oracle(batch, ctx, hkv, dtype, fused):
    bs, dim = 16, 64
    lens = [ctx + 1] * batch  # attend over the context plus the appended token
    seed = batch * 1000 + ctx + hkv
    case = DecodeCase(batch=batch, num_heads=32, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=lens, dtype=dtype, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    new_k = torch.randn(batch, hkv, dim, generator=gen).to(dtype).cuda()
    new_v = torch.randn(batch, hkv, dim, generator=gen).to(dtype).cuda()
    nb = case.cache.layout.num_blocks
    slots = [int(oracle.slot_mapping(case.tables_list[b], ctx, 1, bs, nb)[0]) for b in range(batch)]
    k_want, v_want = to_np(case.cache.k), to_np(case.cache.v)
    oracle.write_slots(k_want, v_want, 0, slots, to_np(new_k), to_np(new_v))
    slots_t = torch.tensor(slots, dtype=torch.int32, device="cuda")
    check_device_errors()
    if fused:
        out = paged_decode_attention_append(case.query, new_k, new_v, case.cache, case.tables,
                                            case.lens, slots_t)
    else:
        append_kv(new_k, new_v, case.cache, slots_t)
        out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    torch.cuda.synchronize()
    assert np.array_equal(to_np(case.cache.k), k_want)
    assert np.array_equal(to_np(case.cache.v), v_want)
    want = oracle.paged_decode_attention(to_np(case.query), k_want, v_want, case.kind,
                                         case.tables_list, lens)
    assert_close(out, want, dtype, f"config 2 B{batch} ctx{ctx} Hkv{hkv}")
    assert check_device_errors() == 0


# ------------------------------------------------------------------ config 4

def _rotary_rows(positions, dim, dtype, theta=5e5):
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    angles = torch.tensor(positions, dtype=torch.float64)[:, None] * inv_freq[None, :]
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().to(dtype).cuda(), emb.sin().to(dtype).cuda()


@pytest.mark.parametrize("kernel", ["tcgen05", "mma_sync"])
@pytest.mark.parametrize("rope", [False, True], ids=["append", "rope_append"])
def test_config4_budget_packed_prefill_step_matches_oracle(rope, kernel):
    hq, hkv, dim, bs, dtype = 32, 8, 128, 16, torch.bfloat16
    lens, batches, tables, num_blocks = config4_plan(seed=0)
    assert len(lens) == 24 and len(batches) >= 2
    assert all(sum(e - s for _, s, e in batch) <= 2048 for batch in batches)
    device = torch.device("cuda", torch.cuda.current_device())
    cache = PagedKVCache(num_blocks, bs, hkv, dim, dtype=dtype, device=device)
    cache.k.fill_(float("nan"))  # unwritten slots must never reach an output
    cache.v.fill_(float("nan"))
    k_want, v_want = to_np(cache.k), to_np(cache.v)
    tables_dev = torch.tensor(tables, dtype=torch.int32, device=device)
    gen = torch.Generator().manual_seed(4)
    check_device_errors()
    runs = []
    for batch in batches:
        ids = [rid for rid, _, _ in batch]
        starts = [s for _, s, _ in batch]
        ends = [e for _, _, e in batch]
        total = sum(e - s for s, e in zip(starts, ends))
        q = torch.randn(total, hq, dim, generator=gen).to(dtype).to(device)
        k = torch.randn(total, hkv, dim, generator=gen).to(dtype).to(device)
        v = torch.randn(total, hkv, dim, generator=gen).to(dtype).to(device)
        btab = tables_dev[ids].contiguous()
        starts_t = torch.tensor(starts, dtype=torch.int32, device=device)
        ends_t = torch.tensor(ends, dtype=torch.int32, device=device)
        slots, cu = build_slot_mapping(btab, starts_t, ends_t, block_size=bs,
                                       num_blocks=num_blocks, total_tokens=total)
        slots_want = np.concatenate([oracle.slot_mapping(tables[i], s, e - s, bs, num_blocks)
                                     for i, s, e in zip(ids, starts, ends)])
        assert np.array_equal(slots.cpu().numpy().astype(np.int64), slots_want)
        assert cu.cpu().tolist() == np.concatenate([[0], np.cumsum(
            [e - s for s, e in zip(starts, ends)])]).tolist()
        if rope:
            positions = [p for s, e in zip(starts, ends) for p in range(s, e)]
            cos, sin = _rotary_rows(positions, dim, dtype)
            q_used = rope_append_kv(q, k, v, cos, sin, cache, slots)
            q_np = oracle.rotary_embed(to_np(q), to_np(cos), to_np(sin), "bf16")
            assert np.array_equal(to_np(q_used), q_np), "rotated query differs from the oracle"
            k_np = oracle.rotary_embed(to_np(k), to_np(cos), to_np(sin), "bf16")
        else:
            append_kv(k, v, cache, slots)
            q_used, q_np, k_np = q, to_np(q), to_np(k)
        oracle.write_slots(k_want, v_want, 0, slots_want, k_np, to_np(v))
        out = paged_prefill_attention_varlen(q_used, cache, btab, cu, starts_t, ends_t,
                                             kernel=kernel)
        runs.append((out, q_np, [tables[i] for i in ids], starts, ends))
    torch.cuda.synchronize()
    assert np.array_equal(to_np(cache.k), k_want), "K cache differs from the oracle"
    assert np.array_equal(to_np(cache.v), v_want), "V cache differs from the oracle"
    for j, (out, q_np, tabs, starts, ends) in enumerate(runs):
        want = oracle.paged_prefill_attention_packed(q_np, k_want, v_want, "bf16", tabs, starts,
                                                     ends)
        assert_close(out, want, dtype, f"config-4 budget batch {j} ({kernel})")
    assert check_device_errors() == 0
