"""numpy restatement of the reference's paged KV cache and paged attention.

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA kernels, never shipped in
the product path (see ``oracle/__init__.py``).

Storage convention (same as the reference, ``cache.py:75-94``): one array per
K and V with shape ``[layers, num_blocks, block_size, kv_heads, head_dim]``.
Element kinds:

* ``"f16"`` -- numpy ``float16``;
* ``"bf16"`` -- numpy ``uint16`` holding the raw bfloat16 bit pattern (numpy
  has no bfloat16 type);
* ``"f32"`` -- numpy ``float32``.

All attention math is done in float32, exactly like the reference's
``dense_decode_attention`` (``attention.py:18-36``) which upcasts with
``.float()`` before its einsum/softmax.  The functions return float32; the
reference casts its result back to the query dtype, which the tests model
with a tolerance instead.
"""

from __future__ import annotations

import numpy as np

_KINDS = ("f16", "bf16", "f32")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw bfloat16 bits (uint16) to float32 exactly (bf16 is the top half of f32)."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 bits, round-to-nearest-even (NaN kept quiet)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    bits = values.view(np.uint32)
    rounding = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((bits + rounding) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(values)
    if nan.any():
        out[nan] = ((bits[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return out


def to_f32(values: np.ndarray, kind: str) -> np.ndarray:
    """Convert a stored array of element kind ``kind`` to float32."""
    if kind not in _KINDS:
        raise ValueError(f"unknown element kind {kind!r}")
    if kind == "bf16":
        return bf16_bits_to_f32(values)
    return np.asarray(values).astype(np.float32)


def slot_mapping(block_table, start: int, length: int, block_size: int, num_blocks: int) -> np.ndarray:
    """Physical slot of each logical token ``start .. start+length-1``.

    Follows ``PagedKVCache.slot_mapping`` (reference ``cache.py:113-129``):
    ``slot = table[p // block_size] * block_size + p % block_size`` as int64,
    with the same three ``ValueError`` checks in the same order.
    """
    if start < 0 or length < 0:
        raise ValueError("start and length must be non-negative")
    table = [int(b) for b in block_table]
    if any(not 0 <= b < num_blocks for b in table):
        raise ValueError("block_table contains an invalid physical block id")
    if length and (start + length - 1) // block_size >= len(table):
        raise ValueError("block_table is shorter than the requested range")
    positions = np.arange(start, start + length, dtype=np.int64)
    logical = positions // block_size
    offsets = positions % block_size
    table_arr = np.asarray(table, dtype=np.int64)
    if length == 0:
        return np.zeros(0, dtype=np.int64)
    return table_arr[logical] * block_size + offsets


def write_slots(k_store: np.ndarray, v_store: np.ndarray, layer: int, slots, key: np.ndarray,
                value: np.ndarray) -> None:
    """Scatter ``key``/``value`` ``[T, Hkv, D]`` to physical ``slots`` in place.

    Follows ``PagedKVCache.write_slots`` (reference ``cache.py:156-189``),
    including its slot range check.  The copy is bit-exact (no conversion).
    """
    _, num_blocks, block_size, _, _ = k_store.shape
    slots = np.asarray(slots, dtype=np.int64)
    if key.shape != value.shape or key.ndim != 3:
        raise ValueError("key/value must have the same [T, H, D] shape")
    if slots.ndim != 1 or slots.shape[0] != key.shape[0]:
        raise ValueError("slots must have one entry per key/value token")
    if slots.size and ((slots < 0).any() or (slots >= num_blocks * block_size).any()):
        raise ValueError("slots contain an invalid physical cache position")
    blocks = slots // block_size
    offsets = slots % block_size
    k_store[layer, blocks, offsets] = key
    v_store[layer, blocks, offsets] = value


def _round_to(values: np.ndarray, kind: str) -> np.ndarray:
    """Round float32 to ``kind`` and widen back (what one torch elementwise op stores)."""
    if kind == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(values))
    if kind == "f16":
        return np.asarray(values, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(values, dtype=np.float32)


def rotary_embed(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, kind: str) -> np.ndarray:
    """Rotary embedding of ``x`` ``[T, H, D]`` with per-token ``cos``/``sin`` ``[T, D]``.

    Follows ``_rotate_half`` / ``_apply_rotary`` (reference
    ``hf_benchmark.py:69-85``): ``x * cos + rotate_half(x) * sin`` with
    ``rotate_half(x) = concat(-x[D/2:], x[:D/2])``, evaluated as torch does for a
    16-bit dtype -- each product and the sum computed in float32 and rounded to
    ``kind``.  Inputs and output are stored arrays of element kind ``kind``
    (bfloat16 as raw uint16 bits).
    """
    xf = to_f32(x, kind)
    cf = to_f32(cos, kind)[:, None, :]
    sf = to_f32(sin, kind)[:, None, :]
    half = xf.shape[-1] // 2
    rot = np.concatenate((-xf[..., half:], xf[..., :half]), axis=-1)
    out = _round_to(_round_to(xf * cf, kind) + _round_to(rot * sf, kind), kind)
    if kind == "bf16":
        return f32_to_bf16_bits(out)
    if kind == "f16":
        return out.astype(np.float16)
    return out


def read_tokens(store: np.ndarray, layer: int, block_table, length: int) -> np.ndarray:
    """First ``length`` logical tokens of one request, in order (reference ``cache.py:191-200``)."""
    _, num_blocks, block_size, _, _ = store.shape
    slots = slot_mapping(block_table, 0, length, block_size, num_blocks)
    return store[layer, slots // block_size, slots % block_size]


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    peak = scores.max(axis=-1, keepdims=True)
    weights = np.exp(scores - peak)
    return weights / weights.sum(axis=-1, keepdims=True)


def dense_decode_attention(query: np.ndarray, key: np.ndarray, value: np.ndarray,
                           scale: float | None = None) -> np.ndarray:
    """``softmax(q k^T * scale) v`` in float32 for one request.

    ``query`` ``[Hq, D]`` float32, ``key``/``value`` ``[T, Hkv, D]`` float32.
    Query head ``h`` reads KV head ``h // (Hq // Hkv)``, which is what the
    reference's ``repeat_interleave`` expansion does (``attention.py:9-15``).
    Follows ``dense_decode_attention`` (reference ``attention.py:18-36``).
    """
    num_heads, head_dim = query.shape
    num_kv_heads = key.shape[1]
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    group = num_heads // num_kv_heads
    scale = head_dim ** -0.5 if scale is None else scale
    k = np.repeat(key, group, axis=1).transpose(1, 0, 2)  # [Hq, T, D]
    v = np.repeat(value, group, axis=1).transpose(1, 0, 2)
    scores = np.einsum("hd,htd->ht", query, k) * np.float32(scale)
    probs = _softmax_rows(scores.astype(np.float32))
    return np.einsum("ht,htd->hd", probs, v).astype(np.float32)


def paged_decode_attention(query: np.ndarray, k_store: np.ndarray, v_store: np.ndarray, kind: str,
                           block_tables, context_lens, scale: float | None = None,
                           layer: int = 0) -> np.ndarray:
    """The reference oracle ``paged_decode_attention`` (``attention.py:134-175``).

    ``query`` ``[B, Hq, D]`` stored as ``kind``; returns float32 ``[B, Hq, D]``.
    One request at a time: read its first ``context_lens[b]`` tokens through
    the block table, then run the float32 dense attention.
    """
    q32 = to_f32(query, kind)
    batch = q32.shape[0]
    if len(context_lens) != batch or len(block_tables) != batch:
        raise ValueError("block_tables and context_lens must have one entry per query")
    outputs = []
    for index in range(batch):
        length = int(context_lens[index])
        if length <= 0:
            raise ValueError("context lengths must be positive")
        key = to_f32(read_tokens(k_store, layer, list(block_tables[index]), length), kind)
        value = to_f32(read_tokens(v_store, layer, list(block_tables[index]), length), kind)
        outputs.append(dense_decode_attention(q32[index], key, value, scale))
    return np.stack(outputs)


def paged_prefill_attention(query: np.ndarray, k_store: np.ndarray, v_store: np.ndarray, kind: str,
                            block_tables, query_starts, context_lens, scale: float | None = None,
                            layer: int = 0) -> np.ndarray:
    """Ragged causal prefill attention over the paged cache, float32.

    ``query`` ``[B, Hq, T, D]``; row ``b`` holds the query tokens of logical
    positions ``query_starts[b] .. context_lens[b]-1``.  Query position ``p``
    attends keys ``0..p``.  Padded query rows (``t >= context_lens[b] -
    query_starts[b]``) attend key 0 only.  Follows
    ``paged_prefill_attention_sdpa`` (reference ``attention.py:230-321``):
    its boolean mask ``allow`` (``:310-313``) and its zeroing of keys beyond
    each context (``:301-305``), with SDPA's softmax over allowed keys.
    """
    q32 = to_f32(query, kind)
    batch, num_heads, width, head_dim = q32.shape
    num_kv_heads = k_store.shape[3]
    group = num_heads // num_kv_heads
    scale = head_dim ** -0.5 if scale is None else scale
    out = np.zeros_like(q32)
    for b in range(batch):
        start = int(query_starts[b])
        end = int(context_lens[b])
        if start < 0 or end - start <= 0:
            raise ValueError("prefill ranges must be non-empty and non-negative")
        if end - start > width:
            raise ValueError("query width is smaller than a prefill range")
        key = to_f32(read_tokens(k_store, layer, list(block_tables[b]), end), kind)
        value = to_f32(read_tokens(v_store, layer, list(block_tables[b]), end), kind)
        for h in range(num_heads):
            kh = key[:, h // group, :]
            vh = value[:, h // group, :]
            for t in range(width):
                limit = start + t + 1 if t < end - start else 1
                scores = (kh[:limit] @ q32[b, h, t]) * np.float32(scale)
                probs = _softmax_rows(scores[None, :].astype(np.float32))[0]
                out[b, h, t] = probs @ vh[:limit]
    return out



def paged_prefill_attention_packed(query: np.ndarray, k_store: np.ndarray, v_store: np.ndarray,
                                   kind: str, block_tables, query_starts, context_lens,
                                   scale: float | None = None, layer: int = 0) -> np.ndarray:
    """The same causal prefill for a packed query ``[sum T, Hq, D]``, float32.

    Sequence ``b`` owns the rows ``sum(T[:b]) .. sum(T[:b+1])-1``, its query
    tokens of logical positions ``query_starts[b] .. context_lens[b]-1``; query
    position ``p`` attends keys ``0..p`` (the unpadded rows of
    ``paged_prefill_attention`` above, which follows reference
    ``attention.py:230-321``).  Vectorised per (sequence, KV head) -- one masked
    score matrix for the whole query-head group -- so full-size budget batches
    finish in seconds; ``tests/test_oracle_golden.py`` holds it equal to the
    loop form and to the reference's golden outputs.
    """
    q32 = to_f32(query, kind)
    total, num_heads, head_dim = q32.shape
    num_kv_heads = k_store.shape[3]
    group = num_heads // num_kv_heads
    scale = head_dim ** -0.5 if scale is None else scale
    out = np.zeros_like(q32)
    row = 0
    for b in range(len(query_starts)):
        start, end = int(query_starts[b]), int(context_lens[b])
        length = end - start
        if start < 0 or length <= 0:
            raise ValueError("prefill ranges must be non-empty and non-negative")
        if row + length > total:
            raise ValueError("packed query holds fewer rows than the prefill ranges")
        key = to_f32(read_tokens(k_store, layer, list(block_tables[b]), end), kind)
        value = to_f32(read_tokens(v_store, layer, list(block_tables[b]), end), kind)
        # visible[t, j]: query row t (position start + t) may attend key j
        visible = np.arange(end)[None, :] <= (start + np.arange(length))[:, None]
        for kv in range(num_kv_heads):
            heads = slice(kv * group, (kv + 1) * group)
            q = q32[row:row + length, heads, :]                      # [T, G, D]
            scores = np.einsum("tgd,jd->gtj", q, key[:, kv, :]) * np.float32(scale)
            scores = np.where(visible[None], scores, -np.inf).astype(np.float32)
            probs = _softmax_rows(scores)
            out[row:row + length, heads, :] = np.einsum("gtj,jd->tgd", probs, value[:, kv, :])
        row += length
    return out
