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


_TORCH_DT = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}


def _noalloc_dt(lib, wid, x, y, stream):
    from burn_rocket_b200 import _lib as L
    code = {"torch.float32": L.DTYPE_F32, "torch.float16": L.DTYPE_F16, "torch.bfloat16": L.DTYPE_BF16}
    return lib.rb_matmul_w8a8_noalloc(wid, x.data_ptr(), code[str(x.dtype)], x.shape[0], x.shape[1],
                                      y.data_ptr(), code[str(y.dtype)], stream)


def _same_bits(a, b):
    import torch
    return torch.equal(a.view(torch.int16) if a.element_size() == 2 else a.view(torch.int32),
                       b.view(torch.int16) if b.element_size() == 2 else b.view(torch.int32))


@pytest.mark.parametrize("x_dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("y_dt", ["f32", "f16", "bf16"])
def test_noalloc_dtypes_match_allocating_entry(rb, orc, x_dt, y_dt):
    """Every input/output dtype pair: bit-identical to rb_matmul."""
    import torch
    from burn_rocket_b200 import _lib as L
    lib = L.load()
    n, k, m = 384, 1152, 517
    rng = np.random.default_rng(77)
    codes, ws = orc.quantize_weight_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wid = rb.pack_qat(codes, ws, n, k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().to(getattr(torch, _TORCH_DT[x_dt]))
    ydt = getattr(torch, _TORCH_DT[y_dt])
    want = rb.matmul(x, wid, out_dtype=ydt)
    got = torch.full((m, n), float("nan"), device="cuda", dtype=ydt)
    assert _noalloc_dt(lib, wid.id, x, got, torch.cuda.current_stream().cuda_stream) == 0, L.last_error()
    torch.cuda.synchronize()
    rb.check_device_errors()
    assert _same_bits(got, want)


def test_noalloc_fused_gelu_and_output_grid(rb, orc):
    """A weight with a fused GELU (f16 out) and one with a calibrated output
    grid (out_scale != 0): bit-identical to rb_matmul; the GELU weight rejects
    a non-f16 output like rb_matmul does."""
    import torch
    from burn_rocket_b200 import _lib as L
    lib = L.load()
    n, k, m = 256, 1152, 300
    rng = np.random.default_rng(78)
    codes, ws = orc.quantize_weight_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().half()

    gelu = rb.pack_qat(codes, ws, n, k)
    rb.set_weight_activation(gelu, "gelu_tanh")
    want = rb.matmul(x, gelu, out_dtype=torch.float16)
    got = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    assert _noalloc_dt(lib, gelu.id, x, got, stream) == 0, L.last_error()
    torch.cuda.synchronize()
    assert _same_bits(got, want)
    bad = torch.zeros(m, n, device="cuda")
    assert _noalloc_dt(lib, gelu.id, x, bad, stream) == L.RB_E_SHAPE
    assert "fused activation" in L.last_error()

    grid = rb.pack_qat(codes, ws, n, k, in_scale=0.0, out_scale=0.05)
    want = rb.matmul(x, grid, out_dtype=torch.float32)
    got = torch.full((m, n), float("nan"), device="cuda")
    assert _noalloc_dt(lib, grid.id, x, got, stream) == 0, L.last_error()
    torch.cuda.synchronize()
    rb.check_device_errors()
    assert _same_bits(got, want)


def test_noalloc_graph_capture_replays(rb, orc):
    """The use it exists for: one eager call, then the same call captured in
    a CUDA graph on a side stream and replayed on new activations, each
    replay bit-identical to rb_matmul on those activations."""
    import torch
    from burn_rocket_b200 import _lib as L
    lib = L.load()
    n, k, m = 1152, 1152, 1000
    rng = np.random.default_rng(79)
    codes, ws = orc.quantize_weight_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wid = rb.pack_qat(codes, ws, n, k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().half()
    y = torch.empty(m, n, device="cuda", dtype=torch.float16)
    assert _noalloc_dt(lib, wid.id, x, y, torch.cuda.current_stream().cuda_stream) == 0, L.last_error()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            assert _noalloc_dt(lib, wid.id, x, y, side.cuda_stream) == 0, L.last_error()
    for rep in range(2):
        x.copy_(torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).half())
        graph.replay()
        torch.cuda.synchronize()
        rb.check_device_errors()
        want = rb.matmul(x, wid, out_dtype=torch.float16)
        torch.cuda.synchronize()
        assert _same_bits(y, want), f"replay {rep}"
    del graph
