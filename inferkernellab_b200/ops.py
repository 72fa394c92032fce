"""Reference-compatible operators backed by the sm_100a kernels.

Each function keeps the signature, argument meaning, validation order and
exception types of the reference wrapper it replaces, so it can be registered
as a backend next to ``paged_reference`` / ``paged_sdpa`` / ``triton_paged``:

=====================================  ==========================================================
this module                            reference (``src/inferkernellab/``)
=====================================  ==========================================================
``paged_decode_attention``             ``triton_ops.paged_decode_attention_triton`` (:404-478) and
                                       ``..._triton_grouped`` (:481-610)
``append_kv``                          ``append.append_kv_triton`` (:69-106)
``paged_prefill_attention``            ``attention.paged_prefill_attention_sdpa`` (:230-321)
``paged_prefill_attention_varlen``     (new) packed ``[sum T, Hq, D]`` form over ``cu_seqlens``
``build_slot_mapping``                 (new) device form of ``PagedKVCache.slot_mapping`` for a batch
``rope_append_kv``                     ``hf_benchmark._apply_rotary`` (:69-85) + ``append_kv_triton``
``paged_decode_attention_append``      (new) the append (+ rotary) above fused into the decode launch
``add_rmsnorm`` / ``silu_mul``         (new) Transformers ``LlamaRMSNorm`` (+ residual add) and the
                                       ``act_fn(gate) * up`` of ``LlamaMLP``, one launch each
=====================================  ==========================================================

All launches go on torch's current CUDA stream through the C ABI in
``_lib``; no torch type crosses it.  There is no CPU or torch fallback: a
missing library, a non-CUDA tensor or an unsupported shape raises.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_DTYPE_CODE = {torch.float16: _lib.B200_F16, torch.bfloat16: _lib.B200_BF16}
# Prefill kernel selector: "auto" takes the tcgen05/TMEM kernel where it applies
# (head_dim 64/128, block_size >= 8), else the mma.sync kernel.
_PREFILL_KERNEL = {"auto": 0, "tcgen05": 1, "mma_sync": 2}
_INDEX_CODE = {torch.int32: _lib.B200_I32, torch.int64: _lib.B200_I64}


def b200_available() -> bool:
    """True when a CUDA device is visible and the library can be loaded."""
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except (OSError, RuntimeError):
        return False
    return True


def _stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _cache_desc(cache) -> _lib.CacheDesc:
    layout = cache.layout
    k, v = cache.k, cache.v
    if k.dtype not in _DTYPE_CODE:
        raise ValueError("the B200 kernels support float16 and bfloat16 caches")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("cache K/V storage must be contiguous")
    if k.device.type != "cuda":
        raise ValueError("the cache must live on a CUDA device")
    return _lib.CacheDesc(k.data_ptr(), v.data_ptr(), layout.num_layers, layout.num_blocks,
                          layout.block_size, layout.num_kv_heads, layout.head_dim,
                          _DTYPE_CODE[k.dtype])


# ----------------------------------------------------------------- workspace

class _Workspaces:
    """Per-(device, stream) decode workspace, zero-filled once and kept.

    The decode kernel's split counters return to zero at the end of every
    launch, so a workspace is only zeroed when it is (re)allocated.  Keeping one
    per stream means launches on different streams never share counters.
    """

    def __init__(self):
        self._lock = threading.Lock()
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}
        self._shape_class: dict[tuple[int, int], tuple] = {}

    def get(self, device: torch.device, stream: int, nbytes: int,
            shape_class: tuple = ()) -> torch.Tensor:
        """Workspace of at least ``nbytes``; re-zeroed when ``shape_class`` changes.

        ``shape_class`` = (group, kv heads, head_dim, block size, dtype): the
        partial-region size depends on it, so a change could leave old partial
        bytes under the split counters (see the header's workspace contract).
        """
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            elif self._shape_class.get(key) != shape_class:
                buf.zero_()
            self._shape_class[key] = shape_class
            return buf

    def reset(self) -> None:
        with self._lock:
            for buf in self._buffers.values():
                buf.zero_()

    def error_words(self):
        with self._lock:
            return list(self._buffers.values())


_WORKSPACES = _Workspaces()


class _ErrorWords:
    """One zeroed device word per device for the append/prefill/metadata kernels."""

    def __init__(self):
        self._lock = threading.Lock()
        self._words: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device) -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            word = self._words.get(index)
            if word is None:
                word = torch.zeros(64, dtype=torch.int32, device=torch.device("cuda", index))
                self._words[index] = word
            return word

    def all(self):
        with self._lock:
            return list(self._words.values())


_ERROR_WORDS = _ErrorWords()


def _read_word(word: torch.Tensor, clear: bool) -> int:
    value = ctypes.c_uint32(0)
    _lib.check(_lib.load().b200_read_error_word(ctypes.c_void_p(word.data_ptr()),
                                                ctypes.byref(value), int(clear),
                                                _stream_ptr(word.device)))
    return int(value.value)


def check_device_errors(clear: bool = True) -> int:
    """Synchronise and return the OR of every decode workspace's device error word.

    Non-zero bits are ``_lib.DEVERR_*``.  A bounded-wait timeout (bits 1, 2, 16)
    means the affected outputs are not valid; in that case the workspaces are
    zeroed again so that stale split counters cannot leak into later calls.
    """
    value = 0
    for buf in _WORKSPACES.error_words() + _ERROR_WORDS.all():
        value |= _read_word(buf, clear)
    if value & (_lib.DEVERR_WAIT_FULL | _lib.DEVERR_WAIT_EMPTY | _lib.DEVERR_DRAIN):
        _WORKSPACES.reset()
    return value


# ------------------------------------------------------------------- decode

def _as_index_tensor(values, device: torch.device) -> torch.Tensor:
    if isinstance(values, list):
        return torch.tensor(values, dtype=torch.int32, device=device)
    return values


def _as_table_tensor(tables, device: torch.device) -> torch.Tensor:
    """Block tables as a 2-D index tensor; ragged Python rows are padded with 0.

    The reference's ``paged_reference`` backend passes one Python list per
    request (``decode.py:400-402``), of different lengths; the Triton backends
    pass a padded ``[B, W]`` tensor.  Entries past a row's context are never
    read, so padding them with block 0 changes nothing.
    """
    if isinstance(tables, (list, tuple)) and tables and all(
            isinstance(row, (list, tuple)) for row in tables):
        width = max(len(row) for row in tables)
        tables = [list(row) + [0] * (width - len(row)) for row in tables]
    return _as_index_tensor(list(tables) if isinstance(tables, tuple) else tables, device)


def paged_decode_attention(query: torch.Tensor, cache, block_tables, context_lens, scale=None,
                           layer: int = 0, *, validate_inputs: bool = True,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Paged decode attention on the sm_100a split-KV kernel.

    Drop-in for ``paged_decode_attention_triton(query, cache, block_tables,
    context_lens, scale=None, layer=0, *, validate_inputs=True)`` (reference
    ``triton_ops.py:404-478``); MHA, GQA and MQA all take the same kernel, so it
    also replaces ``paged_decode_attention_triton_grouped``.  ``out``
    (optional, ``[B, Hq, D]``) receives the result instead of a new tensor.
    """
    if query.ndim != 3 or query.device.type != "cuda":
        raise ValueError("query must be a CUDA tensor with shape [B,H,D]")
    if query.shape[0] <= 0 or query.shape[1] <= 0 or query.shape[2] <= 0:
        raise ValueError("query dimensions must be positive")
    if query.stride(-1) != 1:
        raise ValueError("query must be contiguous in the head_dim dimension")
    block_tables = _as_table_tensor(block_tables, query.device)
    context_lens = _as_index_tensor(context_lens, query.device)
    layout = cache.layout
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    if query.shape[-1] != layout.head_dim:
        raise ValueError("query head_dim does not match cache layout")
    if query.shape[1] % layout.num_kv_heads != 0:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if query.dtype != cache.k.dtype or query.device != cache.k.device:
        raise ValueError("query and cache must have the same dtype and device")
    if block_tables.ndim != 2 or block_tables.shape[0] != query.shape[0]:
        raise ValueError("block_tables must have shape [B, max_blocks]")
    if context_lens.ndim != 1 or context_lens.shape[0] != query.shape[0]:
        raise ValueError("context_lens must have shape [B]")
    if block_tables.device != query.device or context_lens.device != query.device:
        raise ValueError("block_tables and context_lens must be on the query device")
    if block_tables.dtype not in _INDEX_CODE:
        raise ValueError("block_tables must use int32 or int64")
    if context_lens.dtype not in _INDEX_CODE:
        raise ValueError("context_lens must use int32 or int64")
    if block_tables.shape[1] <= 0:
        raise ValueError("block_tables must contain at least one logical block")
    lib = _lib.load()
    stream = _stream_ptr(query.device)
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if not context_lens.is_contiguous():
        context_lens = context_lens.contiguous()
    if validate_inputs:
        flags = torch.empty(3, dtype=torch.int32, device=query.device)
        _lib.check(lib.b200_validate_decode_metadata(
            block_tables.data_ptr(), _INDEX_CODE[block_tables.dtype], block_tables.stride(0),
            block_tables.shape[1], context_lens.data_ptr(), _INDEX_CODE[context_lens.dtype],
            query.shape[0], layout.block_size, layout.num_blocks, flags.data_ptr(), stream))
        bad_len, too_long, bad_block = (bool(x) for x in flags.tolist())
        if bad_len:
            raise ValueError("context lengths must be positive")
        if too_long:
            raise ValueError("context length exceeds block table capacity")
        if bad_block:
            raise ValueError("block table contains an invalid physical block id")
    if query.stride(0) % 2 or query.stride(1) % 2 or query.data_ptr() % 4:
        query = query.contiguous()
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    elif (out.shape != query.shape or out.dtype != query.dtype or out.stride(-1) != 1
          or out.stride(0) % 4 or out.stride(1) % 4 or out.data_ptr() % 8):
        raise ValueError("out must match the query shape and dtype, with rows 8-byte aligned")
    desc = _cache_desc(cache)
    args = _lib.DecodeArgs(
        query.shape[0], query.shape[1], block_tables.shape[1], layer,
        query.stride(0), query.stride(1), out.stride(0), out.stride(1), block_tables.stride(0),
        _INDEX_CODE[block_tables.dtype], _INDEX_CODE[context_lens.dtype],
        float(scale) if scale is not None else layout.head_dim ** -0.5)
    need = lib.b200_paged_decode_workspace_bytes(ctypes.byref(desc), ctypes.byref(args))
    if need == 0:
        _lib.check(_lib.B200_ERR_INVALID if _lib.last_error() else _lib.B200_ERR_CUDA)
    ws = _WORKSPACES.get(query.device, stream.value or 0, need,
                         (query.shape[1] // layout.num_kv_heads, layout.num_kv_heads,
                          layout.head_dim, layout.block_size, query.dtype))
    _lib.check(lib.b200_paged_decode(ctypes.byref(desc), ctypes.byref(args), query.data_ptr(),
                                     block_tables.data_ptr(), context_lens.data_ptr(),
                                     out.data_ptr(), ws.data_ptr(), ws.numel(), stream))
    return out


def _rows16(t: torch.Tensor) -> bool:
    """Rows start on 16-byte boundaries (the fused append moves 16-byte vectors)."""
    return (t.stride(-1) == 1 and all(st % 8 == 0 for st in t.stride()[:-1])
            and t.data_ptr() % 16 == 0)


def paged_decode_attention_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                  cache, block_tables: torch.Tensor, context_lens: torch.Tensor,
                                  slots: torch.Tensor, *, cos: torch.Tensor | None = None,
                                  sin: torch.Tensor | None = None, scale=None, layer: int = 0,
                                  out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step's append and attention in one launch.

    Equivalent to ``rope_append_kv(query, key, value, cos, sin, cache, slots,
    layer)`` (or ``append_kv(key, value, cache, slots, layer)`` when ``cos`` and
    ``sin`` are None) followed by ``paged_decode_attention(rotated_query, cache,
    block_tables, context_lens, scale, layer, validate_inputs=False)`` -- the
    same cache bits and the same attention output -- with the new token's K/V
    written by the attention kernel itself just before it loads the tile that
    holds it (reference ``hf_benchmark.py:69-85`` rotary, ``append.py:69-106``
    append, ``triton_ops.py:404-478`` decode).  Each request's new token must be
    its last context position (``context_lens[b] - 1``).  ``query`` ``[B, Hq, D]``
    (un-rotated when ``cos``/``sin`` are given), ``key``/``value`` ``[B, Hkv, D]``
    (strided views allowed), ``cos``/``sin`` ``[B, D]``, ``slots`` ``[B]``
    int32/int64 (negative: no append for that request).
    """
    if query.ndim != 3 or query.device.type != "cuda":
        raise ValueError("query must be a CUDA tensor with shape [B,H,D]")
    batch, heads, dim = query.shape
    layout = cache.layout
    if key.shape != (batch, layout.num_kv_heads, dim) or value.shape != key.shape:
        raise ValueError("key/value must have shape [B, Hkv, D] matching the cache")
    if dim != layout.head_dim or heads % layout.num_kv_heads != 0:
        raise ValueError("query shape does not match the cache layout")
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    device, dtype = query.device, cache.k.dtype
    for t in (query, key, value):
        if t.dtype != dtype or t.device != device:
            raise ValueError("query/key/value must have the cache dtype and device")
    rope = cos is not None or sin is not None
    if rope:
        if cos is None or sin is None:
            raise ValueError("cos and sin must be given together")
        cos = cos.reshape(-1, dim)
        sin = sin.reshape(-1, dim)
        if cos.shape[0] != batch or sin.shape[0] != batch:
            raise ValueError("cos/sin must hold one [D] row per request")
        if cos.dtype != dtype or sin.dtype != dtype or cos.device != device or sin.device != device:
            raise ValueError("cos/sin must have the cache dtype and device")
        cos, sin = (t if _rows16(t) else t.contiguous() for t in (cos, sin))
    if slots.numel() != batch or slots.dtype not in _INDEX_CODE or slots.device != device:
        raise ValueError("slots must be one int32/int64 entry per request on the query device")
    block_tables = _as_table_tensor(block_tables, device)
    context_lens = _as_index_tensor(context_lens, device)
    if block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError("block_tables must have shape [B, max_blocks]")
    if context_lens.ndim != 1 or context_lens.shape[0] != batch:
        raise ValueError("context_lens must have shape [B]")
    if block_tables.dtype not in _INDEX_CODE or context_lens.dtype not in _INDEX_CODE:
        raise ValueError("block_tables and context_lens must use int32 or int64")
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if not context_lens.is_contiguous():
        context_lens = context_lens.contiguous()
    slots = slots.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    key, value = (t if _rows16(t) else t.contiguous() for t in (key, value))
    # With rope the kernel stages the rotated query in `out` with 16-byte vectors.
    if rope:
        if not _rows16(query):
            query = query.contiguous()
    elif (query.stride(-1) != 1 or query.stride(0) % 2 or query.stride(1) % 2
            or query.data_ptr() % 4):
        query = query.contiguous()
    if out is None:
        out = torch.empty(query.shape, dtype=dtype, device=device)
    elif (out.shape != query.shape or out.dtype != dtype or out.stride(-1) != 1
          or out.stride(0) % 4 or out.stride(1) % 4 or out.data_ptr() % 8
          or (rope and not _rows16(out))):
        raise ValueError("out must match the query shape and dtype, with rows 8-byte aligned "
                         "(16-byte aligned with cos/sin)")
    lib = _lib.load()
    stream = _stream_ptr(device)
    desc = _cache_desc(cache)
    args = _lib.DecodeArgs(
        batch, heads, block_tables.shape[1], layer, query.stride(0), query.stride(1),
        out.stride(0), out.stride(1), block_tables.stride(0), _INDEX_CODE[block_tables.dtype],
        _INDEX_CODE[context_lens.dtype],
        float(scale) if scale is not None else layout.head_dim ** -0.5)
    fused = _lib.DecodeAppendArgs(
        1 if rope else 0, _INDEX_CODE[slots.dtype], key.stride(0), key.stride(1),
        value.stride(0), value.stride(1), cos.stride(0) if rope else 0,
        sin.stride(0) if rope else 0)
    need = lib.b200_paged_decode_workspace_bytes(ctypes.byref(desc), ctypes.byref(args))
    if need == 0:
        _lib.check(_lib.B200_ERR_INVALID if _lib.last_error() else _lib.B200_ERR_CUDA)
    ws = _WORKSPACES.get(device, stream.value or 0, need,
                         (heads // layout.num_kv_heads, layout.num_kv_heads, layout.head_dim,
                          layout.block_size, dtype))
    _lib.check(lib.b200_paged_decode_append(
        ctypes.byref(desc), ctypes.byref(args), ctypes.byref(fused), query.data_ptr(),
        key.data_ptr(), value.data_ptr(), cos.data_ptr() if rope else None,
        sin.data_ptr() if rope else None, slots.data_ptr(), block_tables.data_ptr(),
        context_lens.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(), stream))
    return out


# -------------------------------------------------------------------- append

def append_kv(key: torch.Tensor, value: torch.Tensor, cache, slots: torch.Tensor,
              layer: int = 0) -> None:
    """Scatter ``[T, Hkv, D]`` K/V into ``cache`` at physical ``slots``, bit-exact.

    Drop-in for ``append_kv_triton(key, value, cache, slots, layer=0)``
    (reference ``append.py:69-106``); ``slots`` may be int32 or int64.  Negative
    slots are skipped (padding).
    """
    if key.shape != value.shape or key.ndim != 3:
        raise ValueError("key/value must have shape [T, Hkv, D]")
    if key.device.type != "cuda" or slots.device != key.device or value.device != key.device:
        raise ValueError("key/value/slots must be on the same CUDA device")
    layout = cache.layout
    if tuple(key.shape[1:]) != (layout.num_kv_heads, layout.head_dim):
        raise ValueError("key/value shape does not match cache layout")
    if slots.numel() != key.shape[0]:
        raise ValueError("slots and key/value token counts must match")
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    if key.dtype != cache.k.dtype or value.dtype != cache.k.dtype:
        raise ValueError("key/value must have the cache dtype")
    if slots.dtype not in _INDEX_CODE:
        raise ValueError("slots must use int32 or int64")
    if key.shape[0] == 0:
        return
    if key.stride(-1) != 1:
        key = key.contiguous()
    if value.stride(-1) != 1:
        value = value.contiguous()
    slots = slots.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    desc = _cache_desc(cache)
    _lib.check(_lib.load().b200_append_kv(
        ctypes.byref(desc), layer, key.data_ptr(), value.data_ptr(), key.shape[0],
        key.stride(0), key.stride(1), value.stride(0), value.stride(1), slots.data_ptr(),
        _INDEX_CODE[slots.dtype], _ERROR_WORDS.get(key.device).data_ptr(),
        _stream_ptr(key.device)))


def rope_append_kv(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   cos: torch.Tensor, sin: torch.Tensor, cache, slots: torch.Tensor,
                   layer: int = 0, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate ``query``/``key`` and append rotated K and V to ``cache`` in one launch.

    ``query`` ``[T, Hq, D]``, ``key``/``value`` ``[T, Hkv, D]``, ``cos``/``sin``
    ``[T, D]`` (the per-token rows of the model's rotary table, cache dtype).
    Returns the rotated query (written to ``out`` when given).  Bit-identical to
    the reference's ``_apply_rotary`` (``hf_benchmark.py:69-85``: rounded torch
    elementwise ``x * cos + rotate_half(x) * sin``) followed by
    ``append_kv_triton(key, value, cache, slots, layer)`` (``append.py:69-106``).
    ``query``/``key``/``value`` may be strided views (for instance slices of one
    fused QKV projection) as long as their last dimension is contiguous.
    """
    if query.ndim != 3 or key.ndim != 3 or value.shape != key.shape:
        raise ValueError("query must be [T, Hq, D] and key/value [T, Hkv, D]")
    device = query.device
    if device.type != "cuda" or any(t.device != device for t in (key, value, cos, sin, slots)):
        raise ValueError("query/key/value/cos/sin/slots must be on the same CUDA device")
    layout = cache.layout
    tokens, heads, dim = query.shape
    if tuple(key.shape) != (tokens, layout.num_kv_heads, layout.head_dim) or dim != layout.head_dim:
        raise ValueError("query/key/value shape does not match cache layout")
    if heads % layout.num_kv_heads != 0:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if dim % 2:
        raise ValueError("head_dim must be even for rotary embeddings")
    cos = cos.reshape(-1, dim)
    sin = sin.reshape(-1, dim)
    if cos.shape[0] != tokens or sin.shape[0] != tokens:
        raise ValueError("cos/sin must hold one [D] row per token")
    if slots.numel() != tokens:
        raise ValueError("slots and query token counts must match")
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    dtype = cache.k.dtype
    if any(t.dtype != dtype for t in (query, key, value, cos, sin)):
        raise ValueError("query/key/value/cos/sin must have the cache dtype")
    if slots.dtype not in _INDEX_CODE:
        raise ValueError("slots must use int32 or int64")
    if out is None:
        out = torch.empty((tokens, heads, dim), dtype=dtype, device=device)
    elif out.shape != query.shape or out.dtype != dtype or out.device != device:
        raise ValueError("out must match query's shape, dtype and device")
    if tokens == 0:
        return out
    query, key, value, out = (t if t.stride(-1) == 1 else t.contiguous()
                              for t in (query, key, value, out))
    cos = cos if cos.stride(-1) == 1 else cos.contiguous()
    sin = sin if sin.stride(-1) == 1 else sin.contiguous()
    slots = slots.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    args = _lib.RopeAppendArgs(tokens, heads, layer, query.stride(0), query.stride(1),
                               key.stride(0), key.stride(1), value.stride(0), value.stride(1),
                               out.stride(0), out.stride(1), cos.stride(0), sin.stride(0),
                               _INDEX_CODE[slots.dtype])
    desc = _cache_desc(cache)
    _lib.check(_lib.load().b200_rope_append_kv(
        ctypes.byref(desc), ctypes.byref(args), query.data_ptr(), key.data_ptr(),
        value.data_ptr(), cos.data_ptr(), sin.data_ptr(), slots.data_ptr(), out.data_ptr(),
        _ERROR_WORDS.get(device).data_ptr(), _stream_ptr(device)))
    return out


# ------------------------------------------------------------- layer helpers

def _rows2d(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.ndim != 2:
        raise ValueError(f"{name} must be a 2-D [rows, cols] tensor")
    return t if t.stride(-1) == 1 else t.contiguous()


def add_rmsnorm(x: torch.Tensor | None, residual: torch.Tensor, weight: torch.Tensor,
                eps: float, *, out: torch.Tensor | None = None,
                residual_out: torch.Tensor | None = None):
    """``LlamaRMSNorm(residual + x)`` in one launch; returns ``(normed, summed)``.

    With ``x`` given, the rounded sum ``residual + x`` is written to
    ``residual_out`` (default: in place into ``residual``) and normalised;
    with ``x=None`` ``residual`` itself is normalised and returned as
    ``summed``.  ``[rows, cols]`` tensors in the weight's 16-bit dtype.
    """
    residual = _rows2d(residual, "residual")
    rows, cols = residual.shape
    device, dtype = residual.device, residual.dtype
    if device.type != "cuda" or dtype not in _DTYPE_CODE:
        raise ValueError("add_rmsnorm needs float16/bfloat16 CUDA tensors")
    if weight.shape != (cols,) or weight.dtype != dtype or weight.device != device:
        raise ValueError("weight must be [cols] with the residual's dtype and device")
    weight = weight.contiguous()
    if x is not None:
        x = _rows2d(x, "x")
        if x.shape != residual.shape or x.dtype != dtype or x.device != device:
            raise ValueError("x must match residual's shape, dtype and device")
        if residual_out is None:
            residual_out = residual
        elif (residual_out.shape != residual.shape or residual_out.dtype != dtype
              or residual_out.stride(-1) != 1):
            raise ValueError("residual_out must match residual")
    if out is None:
        out = torch.empty((rows, cols), dtype=dtype, device=device)
    elif out.shape != (rows, cols) or out.dtype != dtype or out.stride(-1) != 1:
        raise ValueError("out must be a [rows, cols] tensor of the residual's dtype")
    _lib.check(_lib.load().b200_add_rmsnorm(
        x.data_ptr() if x is not None else None, residual.data_ptr(), weight.data_ptr(),
        out.data_ptr(), residual_out.data_ptr() if x is not None else None, rows, cols,
        x.stride(0) if x is not None else 0, residual.stride(0), out.stride(0),
        residual_out.stride(0) if x is not None else 0, float(eps), _DTYPE_CODE[dtype],
        _stream_ptr(device)))
    return out, (residual_out if x is not None else residual)


def silu_mul(gate_up: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up`` for ``gate_up = [gate | up]`` rows ``[rows, 2 * I]``, one launch."""
    gate_up = _rows2d(gate_up, "gate_up")
    rows, width = gate_up.shape
    if width % 2:
        raise ValueError("gate_up must hold [gate | up] halves of equal width")
    if gate_up.device.type != "cuda" or gate_up.dtype not in _DTYPE_CODE:
        raise ValueError("silu_mul needs a float16/bfloat16 CUDA tensor")
    cols = width // 2
    if out is None:
        out = torch.empty((rows, cols), dtype=gate_up.dtype, device=gate_up.device)
    elif out.shape != (rows, cols) or out.dtype != gate_up.dtype or out.stride(-1) != 1:
        raise ValueError("out must be [rows, I] in gate_up's dtype")
    _lib.check(_lib.load().b200_silu_mul(
        gate_up.data_ptr(), out.data_ptr(), rows, cols, gate_up.stride(0), out.stride(0),
        _DTYPE_CODE[gate_up.dtype], _stream_ptr(gate_up.device)))
    return out


# ------------------------------------------------------------------- prefill

def _prefill_index(values, device) -> tuple[torch.Tensor, list[int]]:
    if isinstance(values, torch.Tensor):
        host = values.detach().cpu().tolist()
    else:
        host = [int(v) for v in values]
    return torch.tensor(host, dtype=torch.int64, device=device), host


def _prefill_kernel(kernel: str) -> int:
    if kernel not in _PREFILL_KERNEL:
        raise ValueError(f"kernel must be one of {sorted(_PREFILL_KERNEL)}")
    return _PREFILL_KERNEL[kernel]


def paged_prefill_attention(query: torch.Tensor, cache, block_tables, query_starts, context_lens,
                            *, scale=None, layer: int = 0, kernel: str = "auto",
                            validate_inputs: bool = True) -> torch.Tensor:
    """Ragged causal prefill over the paged cache, padded ``[B, Hq, T, D]`` form.

    Drop-in for ``paged_prefill_attention_sdpa`` (reference ``attention.py:230-321``):
    row ``b`` holds query positions ``query_starts[b] .. context_lens[b]-1``;
    padded rows attend key 0 only, as in the reference mask.  The cache must
    already hold every key of each range.

    ``validate_inputs=True`` (the reference's behaviour) reads the ranges to the
    host -- a synchronisation when they are device tensors -- and raises the
    reference's ``ValueError`` for an empty or negative range, a range wider
    than the query or a context past the block table.  ``False`` skips those
    checks and passes device tensors straight to the kernel with no host
    synchronisation (an invalid range is then computed as an empty one, its rows
    attending key 0 like padding rows, and a context past the block table is cut
    at the table's end).
    """
    if query.ndim != 4:
        raise ValueError("query must be [B,H,T,D]")
    batch, num_heads, query_width, head_dim = query.shape
    layout = cache.layout
    if head_dim != layout.head_dim:
        raise ValueError("query head_dim does not match cache")
    if num_heads % layout.num_kv_heads != 0:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if query.device != cache.k.device or query.device.type != "cuda":
        raise ValueError("query and cache must be on the same device")
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    if isinstance(block_tables, torch.Tensor):
        tables = block_tables.to(device=query.device)
    else:
        tables = _as_table_tensor(block_tables, query.device)
    if tables.ndim != 2 or tables.shape[0] != batch:
        raise ValueError("block_tables must have one row per query batch")
    if tables.dtype not in _INDEX_CODE:
        tables = tables.to(torch.int64)
    device_ranges = (not validate_inputs and isinstance(query_starts, torch.Tensor)
                     and isinstance(context_lens, torch.Tensor))
    if device_ranges:
        starts_t = query_starts.to(device=query.device, dtype=torch.int64)
        ends_t = context_lens.to(device=query.device, dtype=torch.int64)
        if starts_t.shape != (batch,) or ends_t.shape != (batch,):
            raise ValueError("query_starts and context_lens must have one entry per query batch")
    else:
        starts_t, starts = _prefill_index(query_starts, query.device)
        ends_t, ends = _prefill_index(context_lens, query.device)
        if len(starts) != batch or len(ends) != batch:
            raise ValueError("query_starts and context_lens must have one entry per query batch")
        lengths = [e - s for s, e in zip(starts, ends)]
        if any(s < 0 or n <= 0 for s, n in zip(starts, lengths)):
            raise ValueError("prefill ranges must be non-empty and non-negative")
        if max(lengths) > query_width:
            raise ValueError("query width is smaller than a prefill range")
        if -(-max(ends) // layout.block_size) > tables.shape[1]:
            raise ValueError("context length exceeds block table capacity")
    if query.dtype != cache.k.dtype:
        raise ValueError("query and cache must have the same dtype")
    if query.stride(-1) != 1 or query.stride(0) % 2 or query.stride(1) % 2 or query.stride(2) % 2:
        query = query.contiguous()
    tables = tables.contiguous()
    out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    desc = _cache_desc(cache)
    args = _lib.PrefillArgs(
        batch, num_heads, tables.shape[1], layer, 0, query_width, 0,
        query.stride(0), query.stride(1), query.stride(2),
        out.stride(0), out.stride(1), out.stride(2), tables.stride(0),
        _INDEX_CODE[tables.dtype], _lib.B200_I64,
        float(scale) if scale is not None else head_dim ** -0.5, _prefill_kernel(kernel))
    _lib.check(_lib.load().b200_paged_prefill(
        ctypes.byref(desc), ctypes.byref(args), query.data_ptr(), tables.data_ptr(),
        starts_t.contiguous().data_ptr(), ends_t.contiguous().data_ptr(), None, out.data_ptr(),
        _ERROR_WORDS.get(query.device).data_ptr(), _stream_ptr(query.device)))
    return out


def paged_prefill_attention_varlen(query: torch.Tensor, cache, block_tables: torch.Tensor,
                                   cu_seqlens_q: torch.Tensor, query_starts: torch.Tensor,
                                   context_lens: torch.Tensor, *, scale=None, layer: int = 0,
                                   out: torch.Tensor | None = None,
                                   kernel: str = "auto") -> torch.Tensor:
    """Packed ragged causal prefill: ``query`` ``[sum T, Hq, D]``, no padding.

    Sequence ``b`` owns rows ``cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1`` which
    are the query tokens of logical positions ``query_starts[b] ..
    context_lens[b]-1``.  All metadata stays on the device (no host sync);
    ``cu_seqlens_q`` is int32, ``query_starts``/``context_lens`` int32 or int64.
    """
    if query.ndim != 3 or query.device.type != "cuda":
        raise ValueError("query must be a CUDA tensor with shape [T,H,D]")
    total, num_heads, head_dim = query.shape
    layout = cache.layout
    if head_dim != layout.head_dim:
        raise ValueError("query head_dim does not match cache")
    if num_heads % layout.num_kv_heads != 0:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if query.dtype != cache.k.dtype or query.device != cache.k.device:
        raise ValueError("query and cache must have the same dtype and device")
    if not 0 <= layer < layout.num_layers:
        raise IndexError("layer is out of range")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_q.ndim != 1:
        raise ValueError("cu_seqlens_q must be a 1-D int32 tensor")
    batch = cu_seqlens_q.shape[0] - 1
    if batch <= 0 or query_starts.shape != (batch,) or context_lens.shape != (batch,):
        raise ValueError("query_starts and context_lens must have one entry per sequence")
    if query_starts.dtype != context_lens.dtype or query_starts.dtype not in _INDEX_CODE:
        raise ValueError("query_starts and context_lens must share an int32/int64 dtype")
    if block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError("block_tables must have one row per sequence")
    if block_tables.dtype not in _INDEX_CODE:
        raise ValueError("block_tables must use int32 or int64")
    if query.stride(-1) != 1 or query.stride(0) % 2 or query.stride(1) % 2:
        query = query.contiguous()
    block_tables = block_tables.contiguous()
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    desc = _cache_desc(cache)
    args = _lib.PrefillArgs(
        batch, num_heads, block_tables.shape[1], layer, 1, 0, total,
        0, query.stride(1), query.stride(0), 0, out.stride(1), out.stride(0),
        block_tables.stride(0), _INDEX_CODE[block_tables.dtype], _INDEX_CODE[query_starts.dtype],
        float(scale) if scale is not None else head_dim ** -0.5, _prefill_kernel(kernel))
    _lib.check(_lib.load().b200_paged_prefill(
        ctypes.byref(desc), ctypes.byref(args), query.data_ptr(), block_tables.data_ptr(),
        query_starts.contiguous().data_ptr(), context_lens.contiguous().data_ptr(),
        cu_seqlens_q.contiguous().data_ptr(), out.data_ptr(),
        _ERROR_WORDS.get(query.device).data_ptr(), _stream_ptr(query.device)))
    return out


# ------------------------------------------------------------------ metadata

def build_slot_mapping(block_tables: torch.Tensor, starts: torch.Tensor, ends: torch.Tensor, *,
                       block_size: int, num_blocks: int, total_tokens: int,
                       slots_dtype: torch.dtype = torch.int32,
                       with_cu_seqlens: bool = True):
    """Device-built slots of every scheduled token of a batch, plus ``cu_seqlens``.

    For each sequence ``b`` and position ``p`` in ``starts[b] .. ends[b]-1``:
    ``slot = block_tables[b, p // block_size] * block_size + p % block_size``,
    packed in sequence order -- the same numbers the reference's per-request
    ``PagedKVCache.slot_mapping`` + ``torch.cat`` produce (``cache.py:113-129``,
    ``decode.py:330-335``), built in one launch from device-resident tables.
    Positions past the table or with an out-of-range block id get ``-1``.
    Returns ``(slots [total_tokens], cu_seqlens int32 [B+1] or None)``.
    """
    if block_tables.ndim != 2 or block_tables.device.type != "cuda":
        raise ValueError("block_tables must be a 2-D CUDA tensor")
    batch = block_tables.shape[0]
    if starts.shape != (batch,) or ends.shape != (batch,):
        raise ValueError("starts and ends must have one entry per table row")
    if starts.dtype != ends.dtype or starts.dtype not in _INDEX_CODE:
        raise ValueError("starts and ends must share an int32/int64 dtype")
    if block_tables.dtype not in _INDEX_CODE or slots_dtype not in _INDEX_CODE:
        raise ValueError("block_tables and slots must use int32 or int64")
    block_tables = block_tables.contiguous() if block_tables.stride(-1) != 1 else block_tables
    device = block_tables.device
    slots = torch.empty(total_tokens, dtype=slots_dtype, device=device)
    cu = torch.empty(batch + 1, dtype=torch.int32, device=device) if with_cu_seqlens else None
    _lib.check(_lib.load().b200_build_slot_mapping(
        block_tables.data_ptr(), _INDEX_CODE[block_tables.dtype], block_tables.stride(0),
        block_tables.shape[1], starts.contiguous().data_ptr(), ends.contiguous().data_ptr(),
        _INDEX_CODE[starts.dtype], batch, block_size, num_blocks,
        slots.data_ptr() if total_tokens else None, _INDEX_CODE[slots_dtype], total_tokens,
        cu.data_ptr() if cu is not None else None, _ERROR_WORDS.get(device).data_ptr(),
        _stream_ptr(device)))
    return slots, cu
