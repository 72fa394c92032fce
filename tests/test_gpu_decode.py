"""Parity of the sm_100a paged decode kernel with the float32 oracle.

Tolerances (written in tests/helpers.TOL): fp16 atol 2e-3 / rtol 1e-2, bf16 atol
1e-2 / rtol 2e-2 against the float32 restatement of the reference's
paged_decode_attention (attention.py:134-175).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import PagedKVCache, check_device_errors, paged_decode_attention
from tests.helpers import DecodeCase, assert_close, from_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("decode_*.npz")), ids=lambda p: p.stem)
def test_decode_matches_reference_golden(path):
    d = np.load(path)
    kind = str(d["kind"])
    dtype = torch.bfloat16 if kind == "bf16" else torch.float16
    k = from_np(d["k"], kind, "cuda")
    v = from_np(d["v"], kind, "cuda")
    layers, nb, bs, hkv, dim = k.shape
    cache = PagedKVCache(nb, bs, hkv, dim, num_layers=layers, dtype=dtype, device="cuda")
    cache.k.copy_(k)
    cache.v.copy_(v)
    query = from_np(d["query"], kind, "cuda")
    scale = None if np.isnan(d["scale"]) else float(d["scale"])
    out = paged_decode_attention(query, cache, torch.tensor(d["block_tables"], device="cuda"),
                                 torch.tensor(d["context_lens"], device="cuda"), scale=scale,
                                 layer=int(d["layer"]))
    assert out.dtype == dtype and out.shape == query.shape
    assert_close(out, d["out_f32"], dtype, path.stem)
    assert check_device_errors() == 0


SHAPES = [
    # (batch, Hq, Hkv, D, BS, lens)
    (4, 32, 8, 64, 16, [512, 512, 512, 512]),           # config 1 shape
    (3, 8, 8, 128, 16, [1, 63, 64]),                     # MHA, tile edges
    (5, 32, 1, 64, 16, [5, 129, 300, 16, 17]),           # MQA G=32
    (2, 64, 1, 64, 16, [100, 257]),                      # G=64
    (3, 32, 1, 64, 16, [640, 1, 65]),                    # G=32, 10 tiles: one CTA per segment
    (3, 32, 1, 64, 16, [641, 1, 65]),                    # G=32, 11 tiles: split ranges
    (3, 16, 2, 128, 16, [1000, 3, 65]),                  # G=8, D128
    (4, 24, 2, 32, 8, [40, 1, 77, 128]),                 # G=12 (padded M tile), D32
    (2, 4, 2, 16, 8, [19, 23]),                          # the reference Triton test shape
    (3, 8, 4, 64, 32, [31, 32, 95]),                     # BS 32
    (2, 8, 2, 64, 128, [130, 600]),                      # BS 128: pages > tile
    (2, 8, 2, 128, 256, [700, 256]),                     # BS 256
    (2, 6, 3, 32, 4, [5, 41]),                           # BS 4 (no swizzle)
    (1, 4, 4, 64, 2, [9]),                               # BS 2 with 128-byte rows
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}_Hq{s[1]}_Hkv{s[2]}_D{s[3]}_BS{s[4]}")
def test_decode_matches_oracle(shape, dtype):
    batch, hq, hkv, dim, bs, lens = shape
    case = DecodeCase(batch=batch, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=lens, dtype=dtype, seed=sum(map(ord, str(shape))) & 0xFFFF)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    assert_close(out, case.oracle(), dtype, str(shape))


@pytest.mark.parametrize("hq,hkv,dim,ctx", [(32, 1, 128, 32768), (64, 1, 64, 32768),
                                             (32, 8, 128, 8192), (8, 2, 32, 8192),
                                             (16, 16, 16, 8192)],
                         ids=["G32_D128", "G64_D64", "G4_D128", "G4_D32", "G1_D16"])
def test_decode_long_request_merges_many_pieces(hq, hkv, dim, ctx):
    """One long request: each segment is cut into ~20-45 split pieces (the split
    size follows the longest segment), so the merge runs many batches
    (transposed variants: lse and partial O loaded together, 16 / outputs-per-
    thread pieces per batch) or, for G > 16 at 32768 tokens, more pieces than
    one 32-piece chunk of lse in shared memory."""
    case = DecodeCase(batch=1, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=16,
                      lens=[ctx], dtype=torch.bfloat16, seed=hq * 131 + dim)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    assert_close(out, case.oracle(), torch.bfloat16, f"Hq{hq} Hkv{hkv} D{dim} ctx{ctx}")
    assert check_device_errors() == 0


@pytest.mark.parametrize("batch", [150, 400], ids=["whole_segments", "split_ranges"])
def test_decode_many_short_segments(batch):
    """Short requests (at most 10 tiles of 32 tokens each at Hkv 2, D 64): with a CTA
    per segment every request runs unsplit, CTA b on request b; with more segments
    than CTAs the kernel falls back to equal split ranges.  Both must match."""
    rng = np.random.default_rng(batch)
    lens = rng.integers(1, 321, size=batch).tolist()
    case = DecodeCase(batch=batch, num_heads=8, num_kv_heads=2, head_dim=64, block_size=16,
                      lens=lens, dtype=torch.bfloat16, seed=batch)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    assert_close(out, case.oracle(), torch.bfloat16, f"batch {batch}")
    assert check_device_errors() == 0


@pytest.mark.parametrize("table_dtype", [torch.int32, torch.int64])
def test_decode_int64_metadata_layer_and_scale(table_dtype):
    case = DecodeCase(batch=3, num_heads=16, num_kv_heads=4, head_dim=64, block_size=16,
                      lens=[70, 1, 333], dtype=torch.bfloat16, layers=3, layer=2,
                      table_dtype=table_dtype, width=30, seed=3)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens, scale=0.07,
                                 layer=2)
    assert_close(out, case.oracle(scale=0.07), torch.bfloat16, "layer2")


def test_decode_ragged_long_config3_subset():
    """Config 3's shape (D128 bf16, Hq32/Hkv8, contexts up to 8192), checked on a subset."""
    gen = torch.Generator().manual_seed(33)
    lens = torch.randint(1, 8193, (16,), generator=gen).tolist()
    lens[0], lens[1] = 8192, 1
    case = DecodeCase(batch=16, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
                      lens=lens, dtype=torch.bfloat16, seed=34)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    assert_close(out, case.oracle(), torch.bfloat16, "config3 subset")


# (Hq, Hkv, D, BS): kv heads per tile 1, 2 (4 heads x 32 tokens needs BS >= 32) and 4.
HEAD_GROUP_SHAPES = [(8, 2, 64, 16), (8, 2, 64, 32), (32, 8, 128, 16)]


@pytest.mark.parametrize("hq,hkv,dim,bs", HEAD_GROUP_SHAPES, ids=["HB1", "HB2", "HB4"])
def test_decode_never_reads_unwritten_nan_slots(hq, hkv, dim, bs):
    case = DecodeCase(batch=3, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=[7, 16, 45], dtype=torch.float16, nan_fill=True,
                      width=-(-45 // bs) + 1, seed=5)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    assert torch.isfinite(out).all()
    assert_close(out, case.oracle(), torch.float16, "nan-poisoned cache")


def test_decode_rejects_invalid_metadata():
    cache = PagedKVCache(8, 8, 2, 16, dtype=torch.float16, device="cuda")
    query = torch.randn(1, 4, 16, device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="positive"):
        paged_decode_attention(query, cache, torch.tensor([[0]], dtype=torch.int32, device="cuda"),
                               torch.tensor([0], dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError, match="physical block"):
        paged_decode_attention(query, cache, torch.tensor([[8]], dtype=torch.int32, device="cuda"),
                               torch.tensor([1], dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError, match="capacity"):
        paged_decode_attention(query, cache, torch.tensor([[1]], dtype=torch.int32, device="cuda"),
                               torch.tensor([9], dtype=torch.int32, device="cuda"))
    with pytest.raises(IndexError):
        paged_decode_attention(query, cache, [[1]], [1], layer=1)
    with pytest.raises(ValueError, match="divisible"):
        paged_decode_attention(torch.randn(1, 3, 16, device="cuda", dtype=torch.float16), cache,
                               [[1]], [1])
    with pytest.raises(ValueError, match="dtype"):
        paged_decode_attention(query.bfloat16(), cache, [[1]], [1])


@pytest.mark.parametrize("hq,hkv,dim,bs", HEAD_GROUP_SHAPES, ids=["HB1", "HB2", "HB4"])
def test_decode_masks_invalid_blocks_without_validation(hq, hkv, dim, bs):
    """validate_inputs=False mirrors the reference kernels: bad pages are skipped."""
    case = DecodeCase(batch=2, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=[40, 40], dtype=torch.float16, seed=9)
    tables = case.tables.clone()
    tables[1, 1] = case.cache.layout.num_blocks + 5  # tokens bs..2bs-1 of request 1 are skipped
    out = paged_decode_attention(case.query, case.cache, tables, case.lens, validate_inputs=False)
    keep = [[t for t in range(40) if not bs <= t < 2 * bs]]
    from tests.helpers import to_np
    k = oracle.read_tokens(to_np(case.cache.k), 0, case.tables_list[1], 40)[keep[0]]
    v = oracle.read_tokens(to_np(case.cache.v), 0, case.tables_list[1], 40)[keep[0]]
    want = oracle.dense_decode_attention(to_np(case.query[1]).astype(np.float32),
                                         k.astype(np.float32), v.astype(np.float32))
    assert_close(out[1:2], want[None], torch.float16, "masked page")
    assert_close(out[:1], case.oracle()[:1], torch.float16, "unaffected request")
    assert check_device_errors() & 8  # DEVERR_BAD_BLOCK reported


def test_decode_lists_are_accepted_and_out_is_reused():
    case = DecodeCase(batch=2, num_heads=4, num_kv_heads=2, head_dim=32, block_size=8,
                      lens=[19, 23], dtype=torch.float16, seed=2)
    out = torch.empty_like(case.query)
    got = paged_decode_attention(case.query, case.cache, case.tables_list, case.lens_list, out=out)
    assert got.data_ptr() == out.data_ptr()
    assert_close(out, case.oracle(), torch.float16, "list metadata")


def test_decode_repeated_calls_are_deterministic_and_keep_workspace_clean():
    case = DecodeCase(batch=6, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
                      lens=[3000, 17, 2048, 1, 900, 4095], dtype=torch.bfloat16, seed=4)
    first = paged_decode_attention(case.query, case.cache, case.tables, case.lens,
                                   validate_inputs=False)
    for _ in range(5):
        again = paged_decode_attention(case.query, case.cache, case.tables, case.lens,
                                       validate_inputs=False)
        assert torch.equal(first, again)
    assert check_device_errors() == 0
    assert_close(first, case.oracle(), torch.bfloat16, "repeat")


def test_decode_on_side_stream():
    case = DecodeCase(batch=2, num_heads=8, num_kv_heads=8, head_dim=64, block_size=16,
                      lens=[100, 200], dtype=torch.float16, seed=8)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = paged_decode_attention(case.query, case.cache, case.tables, case.lens,
                                     validate_inputs=False)
    torch.cuda.current_stream().wait_stream(side)
    assert_close(out, case.oracle(), torch.float16, "side stream")


def test_decode_workspace_survives_changing_batch_and_shape_class():
    """One workspace, calls with growing/shrinking batches and different head
    groupings in a row: split counters must never see stale partial bytes."""
    plan = [
        (6, 32, 8, 128, [3000, 17, 2048, 1, 900, 4095]),
        (16, 32, 8, 128, [8192, 1] + [500 + 431 * i for i in range(14)]),
        (3, 32, 8, 128, [7000, 64, 65]),
        (5, 32, 1, 64, [600, 5, 1200, 33, 2]),
        (40, 32, 8, 128, [97 * (i + 1) for i in range(40)]),
        (2, 32, 8, 128, [5000, 4999]),
    ]
    for i, (batch, hq, hkv, dim, lens) in enumerate(plan):
        case = DecodeCase(batch=batch, num_heads=hq, num_kv_heads=hkv, head_dim=dim,
                          block_size=16, lens=lens, dtype=torch.bfloat16, seed=100 + i)
        out = paged_decode_attention(case.query, case.cache, case.tables, case.lens,
                                     validate_inputs=False)
        assert_close(out, case.oracle(), torch.bfloat16, f"plan step {i}")
    assert check_device_errors() == 0
