"""The allocation-free decode entry point, called through the C ABI.

``b200_paged_decode_noalloc`` serves callers that cannot allocate device memory
while attention runs (a plugin or custom operator inside a host framework that
owns every buffer, or code held to a fixed memory budget): they pass inputs and
outputs only, and the kernel's split scratch comes from the library's static
8 MiB device array.  These tests check it against the workspace entry point
(``b200_paged_decode`` via ``paged_decode_attention``) within the decode
tolerances, on two calls in a row, and that an over-size shape is refused.

This file is collected last on purpose, and it passes both alone in a fresh
process and after the rest of the suite.
"""

import ctypes

import pytest
import torch

from inferkernellab_b200 import _lib, paged_decode_attention
from inferkernellab_b200.ops import _cache_desc
from tests.helpers import TOL, DecodeCase

pytestmark = pytest.mark.gpu


def _noalloc(case: DecodeCase, out: torch.Tensor, scale: float) -> int:
    query, tables, lens = case.query, case.tables, case.lens
    desc = _cache_desc(case.cache)
    args = _lib.DecodeArgs(query.shape[0], query.shape[1], tables.shape[1], case.layer,
                           query.stride(0), query.stride(1), out.stride(0), out.stride(1),
                           tables.stride(0), _lib.B200_I32, _lib.B200_I32, scale)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.load().b200_paged_decode_noalloc(ctypes.byref(desc), ctypes.byref(args),
                                                 query.data_ptr(), tables.data_ptr(),
                                                 lens.data_ptr(), out.data_ptr(), stream)


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
                                  validate_inputs=False).float()
    tol = TOL[dtype]
    for call in range(2):
        out = torch.full_like(case.query, float("nan"))
        rc = _noalloc(case, out, scale)
        assert rc == _lib.B200_OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), want, atol=tol["atol"], rtol=tol["rtol"]), \
            f"call {call}: max |diff| {(out.float() - want).abs().max().item():.3e}"


def test_noalloc_rejects_shapes_beyond_its_scratch():
    case = DecodeCase(batch=2, num_heads=64, num_kv_heads=1, head_dim=128, block_size=16,
                      lens=[100, 200], dtype=torch.bfloat16, seed=5)
    out = torch.empty_like(case.query)
    rc = _noalloc(case, out, 128 ** -0.5)
    assert rc == _lib.B200_ERR_WORKSPACE
    assert "8 MiB" in _lib.last_error()
