"""Failure detection on the device, without a GPU fault.

Every pipeline wait in the kernels is bounded: a wait that runs out flags the
engine's error word and the kernel returns. rb_selftest_wait_timeout runs that
same wait on a barrier nothing arrives on; the host then sees RB_E_DEVICE
naming the wait timeout, and the context keeps working afterwards.
"""
import ctypes as C
import math

import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(rb):
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    waited = C.c_int64(-1)
    rc = lib.rb_selftest_wait_timeout(20_000_000, C.byref(waited))  # 20 ms
    assert rc == L.RB_E_DEVICE
    assert "wait-timeout" in L.last_error()
    assert 20_000 <= waited.value < 2_000_000, waited.value  # microseconds: ran out, did not hang
    # The error word was read and cleared; the device keeps working.
    rb.check_device_errors()
    q = torch.randn(200, 2 * 128, device="cuda").half()
    k = torch.randn(200, 128, device="cuda").half()
    v = torch.randn(200, 128, device="cuda").half()
    out = rb.attention(q, k, v, 2, 1, 128, 1 / math.sqrt(128), None, True)
    torch.cuda.synchronize()
    rb.check_device_errors()
    assert torch.isfinite(out.float()).all()


def test_selftest_rejects_unbounded_limits(rb):
    import burn_rocket_b200._lib as L
    lib = L.load()
    assert lib.rb_selftest_wait_timeout(0, None) == L.RB_E_SHAPE
    assert lib.rb_selftest_wait_timeout(5_000_000_000, None) == L.RB_E_SHAPE
