"""The C-ABI library: it loads without a GPU, exports every symbol the header
declares, and rejects bad arguments before touching the device.  No kernel is
launched here."""

import ctypes
import re
from pathlib import Path

import pytest

from inferkernellab_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_paged_attn.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"B200_API\s+[\w\s\*]+?\b(b200_\w+)\s*\(", text)))


def test_library_builds_and_loads():
    from inferkernellab_b200 import build

    build.build()  # no-op when up to date
    lib = _lib.load()
    assert "sm_100a" in _lib.version()
    assert lib is _lib.load()


def test_every_header_symbol_is_exported():
    declared = _declared_symbols()
    assert declared, "no B200_API declarations found in the header"
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS)
    lib = _lib.load()
    for name in declared:
        assert hasattr(lib, name), name


def test_header_cites_reference_interfaces():
    text = HEADER.read_text()
    for cite in ("triton_ops.py:80-167", "append.py:19-106", "attention.py:230-321",
                 "cache.py:113-129"):
        assert cite in text


def _cache(**kw):
    base = dict(k_cache=None, v_cache=None, num_layers=1, num_blocks=4, block_size=16,
                num_kv_heads=2, head_dim=64, dtype=_lib.B200_F16)
    base.update(kw)
    return _lib.CacheDesc(**base)


def _decode_args(**kw):
    base = dict(num_seqs=1, num_q_heads=4, table_width=1, layer=0, q_stride_seq=256,
                q_stride_head=64, out_stride_seq=256, out_stride_head=64, table_stride=1,
                table_dtype=_lib.B200_I32, lens_dtype=_lib.B200_I32, scale=0.125)
    base.update(kw)
    return _lib.DecodeArgs(**base)


@pytest.mark.parametrize("cache_kw,args_kw,status,match", [
    ({"head_dim": 96}, {}, _lib.B200_ERR_UNSUPPORTED, "head_dim"),
    ({"block_size": 12}, {}, _lib.B200_ERR_UNSUPPORTED, "power of two"),
    ({"dtype": 7}, {}, _lib.B200_ERR_UNSUPPORTED, "float16"),
    ({}, {"layer": 1}, _lib.B200_ERR_LAYER, "layer"),
    ({}, {"num_q_heads": 3}, _lib.B200_ERR_INVALID, "divisible"),
    ({}, {"table_width": 0}, _lib.B200_ERR_INVALID, "logical block"),
    ({"num_kv_heads": 1}, {"num_q_heads": 128}, _lib.B200_ERR_UNSUPPORTED, "64 query heads"),
])
def test_decode_rejects_bad_arguments_on_host(cache_kw, args_kw, status, match):
    lib = _lib.load()
    c, a = _cache(**cache_kw), _decode_args(**args_kw)
    rc = lib.b200_paged_decode(ctypes.byref(c), ctypes.byref(a), None, None, None, None, None, 0,
                               None)
    assert rc == status
    assert match in _lib.last_error()
    with pytest.raises(IndexError if status == _lib.B200_ERR_LAYER else ValueError):
        _lib.check(rc)


def test_append_and_prefill_reject_bad_arguments_on_host():
    lib = _lib.load()
    c = _cache()
    assert lib.b200_append_kv(ctypes.byref(c), 3, None, None, 1, 0, 0, 0, 0, None, 0, None,
                              None) == _lib.B200_ERR_LAYER
    assert lib.b200_append_kv(ctypes.byref(c), 0, None, None, 0, 0, 0, 0, 0, None, 0, None,
                              None) == _lib.B200_OK  # zero tokens: nothing to do
    a = _lib.PrefillArgs(num_seqs=1, num_q_heads=4, table_width=1, layer=0, query_layout=2)
    assert lib.b200_paged_prefill(ctypes.byref(c), ctypes.byref(a), None, None, None, None, None,
                                  None, None, None) == _lib.B200_ERR_INVALID
    assert lib.b200_build_slot_mapping(None, 0, 0, 1, None, None, 0, 0, 16, 4, None, 0, 0, None,
                                       None, None) == _lib.B200_ERR_INVALID


def test_product_package_never_touches_the_oracle():
    pkg = ROOT / "inferkernellab_b200"
    for path in pkg.rglob("*.py"):
        text = path.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", text, re.M), path
        assert "oracle." not in text.replace("oracle.py", ""), path
