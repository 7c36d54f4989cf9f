"""rb_matmul_w8a8_noalloc: the W8A8 matmul entry point that allocates nothing.

Callers that cannot allocate device memory mid-work (CUDA-graph capture, fixed
memory budgets, latency-critical paths) use it instead of rb_matmul; it stages
the int8 activation codes in a fixed device array. Its results must equal the
allocating entry point's bit for bit (the W8A8 bar of the other tests), on two
calls in a row since every call reuses the same array. This file is named to
be collected last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(lib, wid, x, y, stream):
    from burn_rocket_b200 import _lib as L
    return lib.rb_matmul_w8a8_noalloc(wid, x.data_ptr(), L.DTYPE_F32, x.shape[0], x.shape[1], y.data_ptr(),
                                      L.DTYPE_F32, stream)


def test_noalloc_matches_allocating_entry_twice(rb, orc):
    import torch
    from burn_rocket_b200 import _lib as L
    lib = L.load()
    n, k = 1152, 1152
    rng = np.random.default_rng(1234)
    codes, ws = orc.quantize_weight_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wid = rb.pack_qat(codes, ws, n, k)
    stream = torch.cuda.current_stream().cuda_stream
    for call, m in enumerate((2394, 517)):  # two calls in a row, different sizes
        x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
        want = rb.matmul(x, wid)
        got = torch.full((m, n), float("nan"), device="cuda")
        rc = _noalloc(lib, wid.id, x, got, stream)
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        rb.check_device_errors()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), f"call {call}"
        assert np.array_equal(w, orc.w8a8_matmul(x.cpu().numpy(), codes, ws))


def test_noalloc_rejects_oversize_requests(rb, orc):
    import torch
    from burn_rocket_b200 import _lib as L
    lib = L.load()
    n, k = 64, 4096
    codes = np.ones((n, k), np.int8)
    wid = rb.pack_qat(codes, np.full(n, 1e-3, np.float32), n, k)
    m = 9000  # 9000 * 4096 B of codes > the 32 MiB scratch
    x = torch.zeros(m, k, device="cuda")
    y = torch.zeros(m, n, device="cuda")
    rc = _noalloc(lib, wid.id, x, y, torch.cuda.current_stream().cuda_stream)
    assert rc == L.RB_E_SHAPE
    assert "no-allocation scratch" in L.last_error()
