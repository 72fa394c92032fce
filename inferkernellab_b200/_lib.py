"""ctypes binding of ``libb200_paged_attn.so`` (C ABI: ``include/b200_paged_attn.h``).

This module is the only place that talks to the shared library.  It mirrors
the header's structs and prototypes and turns status codes into the
exceptions the reference raises (``ValueError`` for bad inputs, ``IndexError``
for the layer, ``RuntimeError`` for an unavailable backend or a CUDA failure --
reference ``triton_ops.py:415-459``).  There is no fallback: if the library is
missing the first call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libb200_paged_attn.so"

B200_F16, B200_BF16 = 0, 1
B200_I32, B200_I64 = 0, 1

B200_OK = 0
B200_ERR_INVALID = -1
B200_ERR_LAYER = -2
B200_ERR_UNSUPPORTED = -3
B200_ERR_WORKSPACE = -4
B200_ERR_CUDA = -5
B200_ERR_DEVICE = -6

DEVERR_WAIT_FULL = 1
DEVERR_WAIT_EMPTY = 2
DEVERR_BAD_SLOT = 4
DEVERR_BAD_BLOCK = 8
DEVERR_DRAIN = 16

#: Every symbol ``include/b200_paged_attn.h`` declares.
EXPORTED_SYMBOLS = (
    "b200_paged_decode_workspace_bytes",
    "b200_paged_decode",
    "b200_paged_decode_noalloc",
    "b200_paged_decode_noalloc_scratch_bytes",
    "b200_paged_decode_noalloc_error_word",
    "b200_append_kv",
    "b200_rope_append_kv",
    "b200_paged_decode_append",
    "b200_add_rmsnorm",
    "b200_silu_mul",
    "b200_tc_selftest",
    "b200_wait_selftest",
    "b200_paged_prefill",
    "b200_build_slot_mapping",
    "b200_validate_decode_metadata",
    "b200_read_error_word",
    "b200_last_error",
    "b200_version",
)


class CacheDesc(ctypes.Structure):
    _fields_ = [
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("num_layers", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("table_width", ctypes.c_int32),
        ("layer", ctypes.c_int32),
        ("q_stride_seq", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("out_stride_seq", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("table_stride", ctypes.c_int64),
        ("table_dtype", ctypes.c_int32),
        ("lens_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
    ]


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("table_width", ctypes.c_int32),
        ("layer", ctypes.c_int32),
        ("query_layout", ctypes.c_int32),
        ("max_query_len", ctypes.c_int32),
        ("total_query_tokens", ctypes.c_int64),
        ("q_stride_seq", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("q_stride_token", ctypes.c_int64),
        ("o_stride_seq", ctypes.c_int64),
        ("o_stride_head", ctypes.c_int64),
        ("o_stride_token", ctypes.c_int64),
        ("table_stride", ctypes.c_int64),
        ("table_dtype", ctypes.c_int32),
        ("index_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("kernel", ctypes.c_int32),
    ]


class DecodeAppendArgs(ctypes.Structure):
    _fields_ = [
        ("rope", ctypes.c_int32),
        ("slots_dtype", ctypes.c_int32),
        ("k_stride_seq", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_stride_seq", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("cos_stride_seq", ctypes.c_int64),
        ("sin_stride_seq", ctypes.c_int64),
    ]


class RopeAppendArgs(ctypes.Structure):
    _fields_ = [
        ("num_tokens", ctypes.c_int64),
        ("num_q_heads", ctypes.c_int32),
        ("layer", ctypes.c_int32),
        ("q_stride_token", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("k_stride_token", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_stride_token", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("q_out_stride_token", ctypes.c_int64),
        ("q_out_stride_head", ctypes.c_int64),
        ("cos_stride_token", ctypes.c_int64),
        ("sin_stride_token", ctypes.c_int64),
        ("slots_dtype", ctypes.c_int32),
    ]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_PROTOTYPES = {
    "b200_paged_decode_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(CacheDesc),
                                                            ctypes.POINTER(DecodeArgs)]),
    "b200_paged_decode": (ctypes.c_int, [ctypes.POINTER(CacheDesc), ctypes.POINTER(DecodeArgs), _vp,
                                         _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "b200_paged_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(CacheDesc),
                                                 ctypes.POINTER(DecodeArgs), _vp, _vp, _vp, _vp,
                                                 _vp]),
    "b200_paged_decode_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "b200_paged_decode_noalloc_error_word": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p)]),
    "b200_append_kv": (ctypes.c_int, [ctypes.POINTER(CacheDesc), _i32, _vp, _vp, _i64, _i64, _i64,
                                      _i64, _i64, _vp, _i32, _vp, _vp]),
    "b200_paged_decode_append": (ctypes.c_int, [ctypes.POINTER(CacheDesc),
                                                ctypes.POINTER(DecodeArgs),
                                                ctypes.POINTER(DecodeAppendArgs), _vp, _vp, _vp,
                                                _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t,
                                                _vp]),
    "b200_rope_append_kv": (ctypes.c_int, [ctypes.POINTER(CacheDesc),
                                           ctypes.POINTER(RopeAppendArgs), _vp, _vp, _vp, _vp,
                                           _vp, _vp, _vp, _vp, _vp]),
    "b200_add_rmsnorm": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                        _i64, ctypes.c_float, _i32, _vp]),
    "b200_silu_mul": (ctypes.c_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "b200_wait_selftest": (ctypes.c_int, [_i64, _i32, _vp, _vp, _vp]),
    "b200_tc_selftest": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp]),
    "b200_paged_prefill": (ctypes.c_int, [ctypes.POINTER(CacheDesc), ctypes.POINTER(PrefillArgs),
                                          _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_build_slot_mapping": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _vp, _i32, _i32, _i32,
                                               _i32, _vp, _i32, _i64, _vp, _vp, _vp]),
    "b200_validate_decode_metadata": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _i32, _i32, _i32,
                                                     _i32, _vp, _vp]),
    "b200_read_error_word": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint32), _i32, _vp]),
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; ``RuntimeError`` if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"B200 CUDA backend is unavailable: {LIB_PATH} is not built "
                "(run `python -m inferkernellab_b200.build`)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def version() -> str:
    return load().b200_version().decode()


def last_error() -> str:
    return load().b200_last_error().decode()


def check(status: int) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if status == B200_OK:
        return
    msg = last_error() or f"b200 status {status}"
    if status in (B200_ERR_INVALID, B200_ERR_UNSUPPORTED):
        raise ValueError(msg)
    if status == B200_ERR_LAYER:
        raise IndexError(msg)
    raise RuntimeError(msg)
