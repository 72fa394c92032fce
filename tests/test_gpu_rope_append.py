"""Parity of the fused rotary + KV append kernel, bit-exact.

``rope_append_kv`` must return the same bits as the reference's
``_apply_rotary`` (hf_benchmark.py:69-85; pinned through tests/golden/rotary.npz
and the oracle's ``rotary_embed``) and leave the cache exactly as rotating with
torch and then appending with ``append_kv`` / ``PagedKVCache.write_slots``
(cache.py:156-189) would.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from inferkernellab_b200 import PagedKVCache, append_kv, check_device_errors, rope_append_kv
from tests.helpers import KIND, from_np, to_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _torch_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def _rotary_table(positions: torch.Tensor, dim: int, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    angles = positions.double()[:, None] * inv_freq[None, :]
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_rope_append_matches_reference_golden(kind):
    d = np.load(GOLDEN / "rotary.npz")
    dtype = torch.float16 if kind == "f16" else torch.bfloat16
    query = from_np(d[f"{kind}_query"], kind, "cuda")
    key = from_np(d[f"{kind}_key"], kind, "cuda")
    cos = from_np(d[f"{kind}_cos"], kind, "cuda")
    sin = from_np(d[f"{kind}_sin"], kind, "cuda")
    tokens, _, dim = query.shape
    hkv = key.shape[1]
    cache = PagedKVCache(16, 8, hkv, dim, num_layers=2, dtype=dtype, device="cuda")
    cache.k.zero_()
    cache.v.zero_()
    gen = torch.Generator().manual_seed(5)
    slots = torch.randperm(16 * 8, generator=gen)[:tokens].cuda()
    value = torch.randn(key.shape, generator=gen).to(dtype).cuda()
    q_out = rope_append_kv(query, key, value, cos, sin, cache, slots, layer=1)
    torch.cuda.synchronize()
    assert np.array_equal(to_np(q_out).view(np.uint16), d[f"{kind}_q_rot"].view(np.uint16))
    flat_k = cache.k[1].reshape(-1, hkv, dim)[slots]
    flat_v = cache.v[1].reshape(-1, hkv, dim)[slots]
    assert np.array_equal(to_np(flat_k).view(np.uint16), d[f"{kind}_k_rot"].view(np.uint16))
    assert torch.equal(flat_v, value)
    assert int(cache.k[0].abs().sum()) == 0  # other layer untouched
    assert check_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64], ids=["i32", "i64"])
@pytest.mark.parametrize("hq,hkv,dim,bs", [(32, 8, 128, 16), (8, 8, 64, 16), (32, 1, 64, 8),
                                           (4, 2, 16, 4), (24, 2, 32, 32)])
def test_rope_append_bit_exact_against_oracle_with_fused_qkv(dtype, slot_dtype, hq, hkv, dim, bs):
    """q/k/v are strided views of one fused projection output, as a model produces them."""
    gen = torch.Generator().manual_seed(hq * 131 + hkv * 7 + dim + bs)
    tokens, nb, layers, layer = 53, 30, 3, 2
    cache = PagedKVCache(nb, bs, hkv, dim, num_layers=layers, dtype=dtype, device="cuda")
    base_k = torch.randn(cache.k.shape, generator=gen).to(dtype)
    base_v = torch.randn(cache.v.shape, generator=gen).to(dtype)
    cache.k.copy_(base_k)
    cache.v.copy_(base_v)
    qkv = (torch.randn(tokens, (hq + 2 * hkv) * dim, generator=gen) * 2).to(dtype).cuda()
    query = qkv[:, : hq * dim].view(tokens, hq, dim)
    key = qkv[:, hq * dim:(hq + hkv) * dim].view(tokens, hkv, dim)
    value = qkv[:, (hq + hkv) * dim:].view(tokens, hkv, dim)
    positions = torch.randint(0, 32768, (tokens,), generator=gen)
    cos, sin = _rotary_table(positions, dim, dtype)
    cos, sin = cos.cuda(), sin.cuda()
    slots = torch.randperm(nb * bs, generator=gen)[:tokens]
    slots[::9] = -1  # padding tokens: not appended
    q_out = rope_append_kv(query, key, value, cos, sin, cache, slots.to(slot_dtype).cuda(),
                           layer=layer)
    torch.cuda.synchronize()
    kind = KIND[dtype]
    # 1) the rotated query equals torch's rounded elementwise rotary (reference math) on the GPU ...
    assert torch.equal(q_out, _torch_rotary(query, cos, sin))
    # 2) ... and the oracle's restatement
    want_q = oracle.rotary_embed(to_np(query), to_np(cos), to_np(sin), kind)
    assert np.array_equal(to_np(q_out).view(np.uint16), want_q.view(np.uint16))
    # 3) the cache equals the oracle's write_slots of the rotated key and the raw value
    keep = (slots >= 0).numpy()
    k_np, v_np = to_np(base_k), to_np(base_v)
    k_rot = oracle.rotary_embed(to_np(key), to_np(cos), to_np(sin), kind)
    oracle.write_slots(k_np, v_np, layer, slots.numpy()[keep], k_rot[keep], to_np(value)[keep])
    assert np.array_equal(to_np(cache.k).view(np.uint16), k_np.view(np.uint16))
    assert np.array_equal(to_np(cache.v).view(np.uint16), v_np.view(np.uint16))
    assert check_device_errors() == 0


def test_rope_append_equals_rotate_then_append_kv():
    """Same cache bits as the unfused path: torch rotary + append_kv."""
    gen = torch.Generator().manual_seed(11)
    dtype, tokens, hq, hkv, dim, bs, nb = torch.bfloat16, 200, 32, 8, 128, 16, 64
    a = PagedKVCache(nb, bs, hkv, dim, dtype=dtype, device="cuda")
    b = PagedKVCache(nb, bs, hkv, dim, dtype=dtype, device="cuda")
    for c in (a, b):
        c.k.zero_()
        c.v.zero_()
    query = torch.randn(tokens, hq, dim, generator=gen).to(dtype).cuda()
    key = torch.randn(tokens, hkv, dim, generator=gen).to(dtype).cuda()
    value = torch.randn(tokens, hkv, dim, generator=gen).to(dtype).cuda()
    cos, sin = _rotary_table(torch.arange(tokens) + 1000, dim, dtype)
    cos, sin = cos.cuda(), sin.cuda()
    slots = torch.randperm(nb * bs, generator=gen)[:tokens].cuda()
    out = torch.empty_like(query)
    got = rope_append_kv(query, key, value, cos, sin, a, slots, out=out)
    assert got.data_ptr() == out.data_ptr()
    append_kv(_torch_rotary(key, cos, sin), value, b, slots)
    torch.cuda.synchronize()
    assert torch.equal(out, _torch_rotary(query, cos, sin))
    assert torch.equal(a.k, b.k) and torch.equal(a.v, b.v)


def test_rope_append_flags_out_of_pool_slots_and_validates():
    cache = PagedKVCache(4, 8, 2, 16, dtype=torch.float16, device="cuda")
    cache.k.zero_()
    cache.v.zero_()
    query = torch.randn(3, 4, 16, device="cuda", dtype=torch.float16)
    key = torch.randn(3, 2, 16, device="cuda", dtype=torch.float16)
    cos = torch.ones(3, 16, device="cuda", dtype=torch.float16)
    sin = torch.zeros(3, 16, device="cuda", dtype=torch.float16)
    check_device_errors()
    out = rope_append_kv(query, key, key, cos, sin, cache, torch.tensor([0, 32, 5], device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(out, query)  # cos = 1, sin = 0 is the identity rotation
    assert torch.equal(cache.k.view(-1, 2, 16)[[0, 5]], key[[0, 2]])
    assert check_device_errors() & 4  # slot 32 is past the pool: DEVERR_BAD_SLOT
    with pytest.raises(ValueError, match="divisible"):
        rope_append_kv(query[:, :3], key, key, cos, sin, cache, torch.tensor([0, 1, 2], device="cuda"))
    with pytest.raises(ValueError, match="dtype"):
        rope_append_kv(query, key, key, cos.bfloat16(), sin, cache,
                       torch.tensor([0, 1, 2], device="cuda"))
    with pytest.raises(ValueError, match="one \\[D\\] row"):
        rope_append_kv(query, key, key, cos[:2], sin[:2], cache,
                       torch.tensor([0, 1, 2], device="cuda"))
    with pytest.raises(IndexError):
        rope_append_kv(query, key, key, cos, sin, cache, torch.tensor([0, 1, 2], device="cuda"),
                       layer=1)
    empty = rope_append_kv(query[:0], key[:0], key[:0], cos[:0], sin[:0], cache,
                           torch.zeros(0, dtype=torch.int64, device="cuda"))
    assert empty.shape == (0, 4, 16)


def test_rope_append_unaligned_views_take_the_scalar_path():
    """Inputs that are not 16-byte aligned give the same bits as aligned ones."""
    gen = torch.Generator().manual_seed(23)
    dtype, tokens, hq, hkv, dim = torch.float16, 31, 8, 2, 64
    a = PagedKVCache(8, 16, hkv, dim, dtype=dtype, device="cuda")
    b = PagedKVCache(8, 16, hkv, dim, dtype=dtype, device="cuda")
    for c in (a, b):
        c.k.zero_()
        c.v.zero_()
    width = (hq + 2 * hkv) * dim
    flat = torch.randn(tokens, width + 1, generator=gen).to(dtype).cuda()
    qkv = flat[:, 1:]  # one-element offset: every row start is misaligned
    query = qkv[:, : hq * dim].view(tokens, hq, dim)
    key = qkv[:, hq * dim:(hq + hkv) * dim].view(tokens, hkv, dim)
    value = qkv[:, (hq + hkv) * dim:].view(tokens, hkv, dim)
    cos, sin = _rotary_table(torch.arange(tokens) * 37, dim, dtype)
    cos, sin = cos.cuda(), sin.cuda()
    slots = torch.randperm(128, generator=gen)[:tokens].cuda()
    got = rope_append_kv(query, key, value, cos, sin, a, slots)
    want = rope_append_kv(query.contiguous(), key.contiguous(), value.contiguous(), cos, sin, b,
                          slots)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and torch.equal(got, _torch_rotary(query, cos, sin))
    assert torch.equal(a.k, b.k) and torch.equal(a.v, b.v)
