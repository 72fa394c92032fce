"""The allocation-free decode entry point, called through the C ABI.

``b200_paged_decode_noalloc`` serves callers that cannot allocate device memory
while attention runs (a plugin or custom operator inside a host framework that
owns every buffer, or code held to a fixed memory budget): they pass inputs and
outputs only, and the kernel's split scratch comes from the library's static
8 MiB device array.  These tests check, on two calls in a row, that it gives
exactly the workspace entry point's output (``b200_paged_decode`` via
``paged_decode_attention``: same kernel, same grid), that both are within the
decode tolerances of the float32 oracle, that the array's error word (read
through ``b200_paged_decode_noalloc_error_word``) stays clear on valid input
and reports a masked out-of-pool block, and that an over-size shape is refused.

This file is collected last on purpose, and it passes both alone in a fresh
process and after the rest of the suite.
"""

import ctypes

import pytest
import torch

from inferkernellab_b200 import _lib, paged_decode_attention
from inferkernellab_b200.ops import _cache_desc
from tests.helpers import DecodeCase, assert_close

pytestmark = pytest.mark.gpu


def _noalloc(case: DecodeCase, out: torch.Tensor, scale: float, tables=None) -> int:
    query, lens = case.query, case.lens
    tables = case.tables if tables is None else tables
    desc = _cache_desc(case.cache)
    args = _lib.DecodeArgs(query.shape[0], query.shape[1], tables.shape[1], case.layer,
                           query.stride(0), query.stride(1), out.stride(0), out.stride(1),
                           tables.stride(0), _lib.B200_I32, _lib.B200_I32, scale)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.load().b200_paged_decode_noalloc(ctypes.byref(desc), ctypes.byref(args),
                                                 query.data_ptr(), tables.data_ptr(),
                                                 lens.data_ptr(), out.data_ptr(), stream)


def _error_word() -> int:
    """Reads (and clears) the static array's error word on the current device."""
    lib = _lib.load()
    addr = ctypes.c_void_p()
    rc = lib.b200_paged_decode_noalloc_error_word(ctypes.byref(addr))
    assert rc == _lib.B200_OK, _lib.last_error()
    assert addr.value
    value = ctypes.c_uint32(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.b200_read_error_word(addr, ctypes.byref(value), 1, stream)
    assert rc == _lib.B200_OK, _lib.last_error()
    return value.value


@pytest.mark.parametrize("shape", [
    # (batch, Hq, Hkv, D, BS, lens, dtype)
    (8, 32, 8, 128, 16, [4000, 1, 77, 2048, 513, 8192, 64, 300], torch.bfloat16),
    (4, 32, 8, 64, 16, [512, 512, 512, 512], torch.float16),
    (3, 32, 1, 64, 16, [900, 17, 1], torch.float16),
])
def test_noalloc_matches_workspace_entry_point_twice(shape):
    batch, hq, hkv, dim, bs, lens, dtype = shape
    lib = _lib.load()
    assert lib.b200_paged_decode_noalloc_scratch_bytes() == 8 << 20
    case = DecodeCase(batch=batch, num_heads=hq, num_kv_heads=hkv, head_dim=dim, block_size=bs,
                      lens=lens, dtype=dtype, seed=batch * 31 + dim)
    scale = dim ** -0.5
    want = paged_decode_attention(case.query, case.cache, case.tables, case.lens,
                                  validate_inputs=False)
    assert_close(want, case.oracle(), dtype, "workspace entry point vs oracle")
    for call in range(2):
        out = torch.full_like(case.query, float("nan"))
        rc = _noalloc(case, out, scale)
        assert rc == _lib.B200_OK, _lib.last_error()
        assert _error_word() == 0, f"call {call}: device error word set"
        assert torch.equal(out, want), \
            f"call {call}: max |diff| {(out.float() - want.float()).abs().max().item():.3e}"
        assert_close(out, case.oracle(), dtype, f"no-alloc call {call} vs oracle")


def test_noalloc_reports_a_masked_block_through_its_error_word():
    case = DecodeCase(batch=2, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
                      lens=[100, 40], dtype=torch.bfloat16, seed=11)
    bad = case.tables.clone()
    bad[1, 0] = case.cache.layout.num_blocks + 3  # outside the pool: masked, flagged
    out = torch.empty_like(case.query)
    assert _noalloc(case, out, 128 ** -0.5, tables=bad) == _lib.B200_OK, _lib.last_error()
    assert _error_word() & _lib.DEVERR_BAD_BLOCK
    # the next call starts from a clear word and request 0 is unaffected
    assert _noalloc(case, out, 128 ** -0.5) == _lib.B200_OK, _lib.last_error()
    assert _error_word() == 0
    assert_close(out, case.oracle(), torch.bfloat16, "no-alloc after a flagged call")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    case = DecodeCase(batch=2, num_heads=64, num_kv_heads=1, head_dim=128, block_size=16,
                      lens=[100, 200], dtype=torch.bfloat16, seed=5)
    out = torch.empty_like(case.query)
    rc = _noalloc(case, out, 128 ** -0.5)
    assert rc == _lib.B200_ERR_WORKSPACE
    assert "8 MiB" in _lib.last_error()
