"""A bounded device wait that runs out, and the context after it.

Every kernel of the library waits on its mbarriers through one bounded wait: it
gives up after a time limit (1 s in the kernels), records
``B200_DEVERR_WAIT_FULL`` in the device error word and raises the CTA's abort
flag, through which the CTA's other waiters leave, so the kernel returns
instead of hanging.  ``b200_wait_selftest`` runs that wait with a short limit
on an mbarrier nobody arrives at (no copy or MMA is in flight), which is how
this test makes a wait run out without faulting or hanging anything.  After
it, a normal decode launch must still be correct.
"""

import ctypes

import pytest
import torch

from inferkernellab_b200 import _lib, check_device_errors, paged_decode_attention
from tests.helpers import DecodeCase, assert_close

pytestmark = pytest.mark.gpu


def _selftest(limit_ns: int, arrive: bool):
    result = torch.zeros(3, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.load().b200_wait_selftest(limit_ns, 1 if arrive else 0, result.data_ptr(),
                                        err.data_ptr(), stream)
    assert rc == _lib.B200_OK, _lib.last_error()
    torch.cuda.synchronize()
    done0, done2, spent = (int(x) & 0xFFFFFFFF for x in result.tolist())
    return done0, done2, spent, int(err.item()) & 0xFFFFFFFF


def test_wait_that_nobody_satisfies_gives_up_and_sets_the_error_bit():
    limit = 200_000  # 200 us
    done0, done2, spent, err = _selftest(limit, arrive=False)
    assert done0 == 0 and done2 == 0  # no wait completed ...
    assert err == _lib.DEVERR_WAIT_FULL  # ... the give-up was recorded once, as WAIT_FULL
    assert limit <= spent < 1_000_000_000  # after the limit, long before the kernels' 1 s


def test_satisfied_wait_completes_without_error():
    done0, done2, _, err = _selftest(200_000, arrive=True)
    assert (done0, done2, err) == (32, 32, 0)


def test_decode_is_correct_after_a_wait_ran_out():
    assert _selftest(100_000, arrive=False)[3] == _lib.DEVERR_WAIT_FULL
    check_device_errors()
    case = DecodeCase(batch=4, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
                      lens=[700, 1, 2049, 130], dtype=torch.bfloat16, seed=3)
    out = paged_decode_attention(case.query, case.cache, case.tables, case.lens)
    torch.cuda.synchronize()
    assert_close(out, case.oracle(), torch.bfloat16, "decode after a timed-out wait")
    assert check_device_errors() == 0


def test_wait_selftest_rejects_out_of_range_limits():
    lib = _lib.load()
    buf = torch.zeros(4, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for bad in (0, 999, 3_000_000_000):
        rc = lib.b200_wait_selftest(bad, 0, buf.data_ptr(), buf[3:].data_ptr(), stream)
        assert rc == _lib.B200_ERR_INVALID
        assert "limit_ns" in _lib.last_error()
