"""Decode with the new token's append (and rotary embedding) fused into the
attention launch, against the unfused calls and the oracle.

The fused call must leave the cache bit-identical to ``rope_append_kv`` /
``append_kv`` (reference hf_benchmark.py:69-85 rotary, append.py:69-106 append)
and give the attention output of ``paged_decode_attention`` on the rotated
query (reference triton_ops.py:404-478), within the decode tolerances of
tests/helpers.TOL against the float32 oracle.
"""

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import (
    append_kv,
    check_device_errors,
    paged_decode_attention,
    paged_decode_attention_append,
    rope_append_kv,
)
from tests.helpers import DecodeCase, assert_close, to_np

pytestmark = pytest.mark.gpu


def _rotary_rows(positions, dim, dtype):
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    angles = torch.tensor(positions, dtype=torch.float64)[:, None] * inv_freq[None, :]
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().to(dtype).cuda(), emb.sin().to(dtype).cuda()


def _setup(shape, dtype, seed, slot_dtype=torch.int32):
    batch, hq, hkv, dim, bs, lens = shape
    case = DecodeCase(batch=batch, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=lens, dtype=dtype, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    # The new token of request b sits at position lens[b] - 1.
    slots = [int(oracle.slot_mapping(case.tables_list[b], n - 1, 1, bs,
                                     case.cache.layout.num_blocks)[0])
             for b, n in enumerate(lens)]
    qkv = torch.randn(batch, (hq + 2 * hkv) * dim, generator=gen).to(dtype).cuda()
    query = qkv[:, : hq * dim].view(batch, hq, dim)
    key = qkv[:, hq * dim:(hq + hkv) * dim].view(batch, hkv, dim)
    value = qkv[:, (hq + hkv) * dim:].view(batch, hkv, dim)
    cos, sin = _rotary_rows([n - 1 for n in lens], dim, dtype)
    return case, query, key, value, cos, sin, torch.tensor(slots, dtype=slot_dtype, device="cuda")


SHAPES = [
    # (batch, Hq, Hkv, D, BS, lens)
    (16, 32, 8, 128, 16, [8192, 1, 77, 2048, 513, 4000, 64, 65, 300, 1000, 17, 129, 3000, 5, 700, 9]),
    (4, 32, 8, 64, 16, [512, 512, 512, 512]),          # config 1 shape
    (3, 8, 8, 128, 16, [1, 63, 64]),                   # MHA, tile edges
    (3, 24, 2, 32, 8, [40, 1, 77]),                    # G = 12 (N = 16 variant)
    (2, 64, 2, 64, 16, [100, 257]),                    # G = 32 (heads as M)
    (2, 64, 1, 128, 16, [300, 31]),                    # G = 64
    (3, 32, 1, 64, 16, [641, 9, 700]),                 # G = 32, split ranges (> 10 tiles)
    (2, 4, 2, 16, 8, [19, 23]),                        # D = 16
    (2, 8, 2, 64, 128, [130, 600]),                    # block size 128
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}_Hq{s[1]}_Hkv{s[2]}_D{s[3]}_BS{s[4]}")
def test_fused_rope_append_decode_matches_unfused(shape, dtype):
    case, query, key, value, cos, sin, slots = _setup(shape, dtype, seed=len(shape[5]) + shape[3])
    ref_cache_k, ref_cache_v = case.cache.k.clone(), case.cache.v.clone()
    out = paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens,
                                        slots, cos=cos, sin=sin)
    fused_k, fused_v = case.cache.k.clone(), case.cache.v.clone()
    # Unfused: rotary + append, then decode on the rotated query.
    case.cache.k.copy_(ref_cache_k)
    case.cache.v.copy_(ref_cache_v)
    q_rot = rope_append_kv(query, key, value, cos, sin, case.cache, slots)
    want = paged_decode_attention(q_rot, case.cache, case.tables, case.lens, validate_inputs=False)
    torch.cuda.synchronize()
    assert torch.equal(fused_k, case.cache.k) and torch.equal(fused_v, case.cache.v)
    assert torch.allclose(out.float(), want.float(), atol=1e-6, rtol=0), \
        f"max |diff| {(out.float() - want.float()).abs().max().item():.3e}"
    case.query = q_rot  # the oracle sees the rotated query and the appended cache
    assert_close(out, case.oracle(), dtype, str(shape))
    assert check_device_errors() == 0


@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
def test_fused_plain_append_decode_matches_append_kv(slot_dtype):
    shape = (6, 32, 8, 128, 16, [3000, 17, 2048, 1, 900, 4095])
    case, query, key, value, _, _, slots = _setup(shape, torch.bfloat16, seed=7,
                                                  slot_dtype=slot_dtype)
    k0, v0 = case.cache.k.clone(), case.cache.v.clone()
    out = paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens,
                                        slots)
    fk, fv = case.cache.k.clone(), case.cache.v.clone()
    case.cache.k.copy_(k0)
    case.cache.v.copy_(v0)
    append_kv(key, value, case.cache, slots)
    want = paged_decode_attention(query, case.cache, case.tables, case.lens, validate_inputs=False)
    torch.cuda.synchronize()
    assert torch.equal(fk, case.cache.k) and torch.equal(fv, case.cache.v)
    assert torch.allclose(out.float(), want.float(), atol=1e-6, rtol=0)


def test_fused_append_skips_negative_and_flags_out_of_pool_slots():
    shape = (3, 8, 2, 64, 16, [40, 70, 5])
    case, query, key, value, cos, sin, slots = _setup(shape, torch.float16, seed=3)
    nb_slots = case.cache.layout.num_blocks * case.cache.layout.block_size
    bad = slots.clone()
    bad[0] = -1            # padding: no append, attention reads the old slot content
    bad[2] = nb_slots + 5  # outside the pool: skipped and flagged
    k0 = case.cache.k.clone()
    check_device_errors()
    paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens, bad,
                                  cos=cos, sin=sin)
    torch.cuda.synchronize()
    flat_new = case.cache.k.view(-1, 2, 64)
    flat_old = k0.view(-1, 2, 64)
    assert torch.equal(flat_new[slots[0]], flat_old[slots[0]])  # untouched
    assert not torch.equal(flat_new[slots[1]], flat_old[slots[1]])  # appended
    assert torch.equal(flat_new[slots[2]], flat_old[slots[2]])
    assert check_device_errors() & 4  # DEVERR_BAD_SLOT


def test_fused_append_validates_arguments():
    shape = (2, 8, 2, 64, 16, [10, 20])
    case, query, key, value, cos, sin, slots = _setup(shape, torch.float16, seed=4)
    with pytest.raises(ValueError, match="together"):
        paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens,
                                      slots, cos=cos)
    with pytest.raises(ValueError, match="key/value"):
        paged_decode_attention_append(query, key[:, :1], value, case.cache, case.tables,
                                      case.lens, slots)
    with pytest.raises(ValueError, match="slots"):
        paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens,
                                      slots[:1])
    with pytest.raises(IndexError):
        paged_decode_attention_append(query, key, value, case.cache, case.tables, case.lens,
                                      slots, layer=1)
