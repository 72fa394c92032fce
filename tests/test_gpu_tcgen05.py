"""The tcgen05 (tensor memory) path: building-block self-test and the tcgen05
prefill kernel against the float32 oracle and the mma.sync kernel.

Tolerances (tests/helpers.TOL) are the north-star ones against the float32
restatement of the reference's paged_prefill_attention_sdpa
(attention.py:230-321): fp16 atol 2e-3 / rtol 1e-2, bf16 atol 1e-2 / rtol 2e-2.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import (
    _lib,
    check_device_errors,
    paged_prefill_attention,
    paged_prefill_attention_varlen,
)
from tests.helpers import KIND, assert_close, to_np
from tests.test_gpu_append_prefill import _prefill_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_tcgen05_selftest_descriptors_and_tmem(dtype):
    """K-major and MN-major 128B-swizzled operands, MMAs into TMEM, tcgen05.ld, and
    the A-from-tensor-memory MMA form with A written by tcgen05.st."""
    gen = torch.Generator().manual_seed(3)
    a = torch.randn(128, 64, generator=gen).to(dtype).cuda()
    b = torch.randn(64, 64, generator=gen).to(dtype).cuda()
    v = torch.randn(64, 128, generator=gen).to(dtype).cuda()
    c1 = torch.full((128, 64), float("nan"), device="cuda")
    c2 = torch.full((128, 128), float("nan"), device="cuda")
    c3 = torch.full((128, 128), float("nan"), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    code = _lib.B200_BF16 if dtype == torch.bfloat16 else _lib.B200_F16
    rc = _lib.load().b200_tc_selftest(a.data_ptr(), b.data_ptr(), v.data_ptr(), c1.data_ptr(),
                                      c2.data_ptr(), c3.data_ptr(), code, err.data_ptr(),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.B200_OK, _lib.last_error()
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    want1 = a.double() @ b.double().T
    want2 = a.double() @ v.double()
    assert torch.allclose(c1.double(), want1, atol=1e-3, rtol=1e-4)
    assert torch.allclose(c2.double(), want2, atol=1e-3, rtol=1e-4)
    assert torch.allclose(c3.double(), want2, atol=1e-3, rtol=1e-4)  # A from tensor memory


CASES = [
    # (Hq, Hkv, D, BS, starts, ends)
    (32, 8, 128, 16, [0, 0, 100], [300, 17, 229]),     # config-4 like, chunk continuation
    (8, 8, 64, 16, [0, 5], [128, 133]),                # MHA, exact 128-row tile
    (32, 1, 64, 16, [0], [150]),                       # MQA
    (8, 2, 128, 256, [0, 200], [513, 300]),            # big pages, 5 query tiles
    (4, 2, 128, 32, [0, 900], [1100, 1000]),           # long prefix: lazy rescale over many tiles
    (6, 3, 64, 8, [10, 0, 3], [43, 9, 260]),           # block size 8
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("cfg", CASES, ids=lambda c: f"Hq{c[0]}_Hkv{c[1]}_D{c[2]}_BS{c[3]}")
def test_tcgen05_prefill_matches_oracle(cfg, dtype):
    hq, hkv, dim, bs, starts, ends = cfg
    cache, tables, query = _prefill_case(dtype, hq, hkv, dim, bs, starts, ends,
                                         seed=sum(ends) + dim)
    out = paged_prefill_attention(query, cache, tables, starts, ends, kernel="tcgen05")
    want = oracle.paged_prefill_attention(to_np(query), to_np(cache.k), to_np(cache.v),
                                          KIND[dtype], tables, starts, ends)
    assert_close(out, want, dtype, str(cfg))
    ref = paged_prefill_attention(query, cache, tables, starts, ends, kernel="mma_sync")
    assert_close(out, to_np(ref.float()), dtype, "vs mma.sync kernel")
    assert check_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_tcgen05_prefill_repeated_calls_are_identical_and_never_time_out(dtype):
    """The kernel's roles hand tiles over through mbarrier phases; a hand-off that
    can run two phases ahead of its waiter hangs that CTA until the bounded wait
    gives up (error bit, garbage rows).  Such races show up only under some
    timings, so the same multi-tile launch is repeated: every output must equal the
    first bit for bit (the per-row arithmetic order is fixed) and no wait may
    time out."""
    hq, hkv, dim, bs, starts, ends = CASES[0]
    cache, tables, query = _prefill_case(dtype, hq, hkv, dim, bs, starts, ends, seed=77)
    check_device_errors()
    first = paged_prefill_attention(query, cache, tables, starts, ends, kernel="tcgen05")
    for _ in range(30):
        out = paged_prefill_attention(query, cache, tables, starts, ends, kernel="tcgen05")
        assert torch.equal(out, first)
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    want = oracle.paged_prefill_attention(to_np(query), to_np(cache.k), to_np(cache.v),
                                          KIND[dtype], tables, starts, ends)
    assert_close(first, want, dtype, "repeated")


def test_tcgen05_prefill_packed_nan_poisoned_cache_and_masked_block():
    """Unwritten slots hold NaN; a bad block id in one table is masked (its keys
    are skipped, its V rows never reach O)."""
    dtype = torch.bfloat16
    starts, ends = [0, 33, 7], [197, 50, 8]
    cache, tables, query = _prefill_case(dtype, 16, 4, 128, 16, starts, ends, seed=91,
                                         nan_fill=True)
    lens = [e - s for s, e in zip(starts, ends)]
    packed = torch.cat([query[b, :, :n].transpose(0, 1) for b, n in enumerate(lens)]).contiguous()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    args = (cache, torch.tensor(tables, dtype=torch.int32, device="cuda"), cu,
            torch.tensor(starts, dtype=torch.int32, device="cuda"),
            torch.tensor(ends, dtype=torch.int32, device="cuda"))
    out = paged_prefill_attention_varlen(packed, *args, kernel="tcgen05")
    assert torch.isfinite(out).all()
    ref = paged_prefill_attention_varlen(packed, *args, kernel="mma_sync")
    assert_close(out, to_np(ref.float()), dtype, "packed vs mma.sync")
    padded = paged_prefill_attention(query, cache, tables, starts, ends, kernel="tcgen05")
    want = oracle.paged_prefill_attention(to_np(query), to_np(cache.k), to_np(cache.v), "bf16",
                                          tables, starts, ends)
    assert_close(padded, want, dtype, "padded vs oracle")
    assert torch.equal(out, torch.cat([padded[b, :, :n].transpose(0, 1)
                                       for b, n in enumerate(lens)]))
    # Mask block 1 of sequence 0 (keys 16..31): both kernels skip those keys.
    bad = torch.tensor(tables, dtype=torch.int32, device="cuda")
    bad[0, 1] = cache.layout.num_blocks + 3
    args_bad = (cache, bad) + args[2:]
    got = paged_prefill_attention_varlen(packed, *args_bad, kernel="tcgen05")
    ref_bad = paged_prefill_attention_varlen(packed, *args_bad, kernel="mma_sync")
    assert torch.isfinite(got).all()
    assert_close(got, to_np(ref_bad.float()), dtype, "masked block")
    assert check_device_errors() & 8


def test_tcgen05_prefill_is_refused_where_it_cannot_run():
    dtype = torch.float16
    cache, tables, query = _prefill_case(dtype, 4, 2, 32, 8, [0], [20], seed=1)
    with pytest.raises(ValueError, match="tcgen05"):
        paged_prefill_attention(query, cache, tables, [0], [20], kernel="tcgen05")
    with pytest.raises(ValueError, match="kernel"):
        paged_prefill_attention(query, cache, tables, [0], [20], kernel="wgmma")
