"""Device parity of the quantised matmuls against the CPU oracle, through the
C ABI (librocket_b200.so).

Bars (north star): the Q8_0 dequantisation and the W8A8 int32 accumulators are
bit-exact; W8A8 outputs are bit-exact too (the epilogue is a fixed sequence of
f32 roundings); Q8_0 GEMM outputs reach cosine >= 0.9999 and a max error of at
most 1e-2 of the output's max magnitude against the reference f32 path
(f64-accumulated product with the exactly dequantised weight).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_REL = 1e-2


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def max_rel(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max() / (np.abs(want).max() + 1e-30))


def q8_weight(orc, n, k, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * std).astype(np.float32)
    codes, scales = orc.q8_0_quantize(w)
    return w, codes, scales


# ------------------------------------------------------------------ Q8_0 codec on device
@pytest.mark.parametrize("n,k", [(64, 32), (3072, 1024), (130, 96)])
def test_q8_0_device_encode_and_dequant_bit_exact(rb, orc, n, k):
    import torch
    w, codes, scales = q8_weight(orc, n, k, seed=n * 7 + k)
    deq = orc.q8_0_dequant(codes, scales)
    # GGUF block ingest
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), n, k)
    got = rb.q8_0_dequant(wid, "f32").cpu().numpy()
    assert np.array_equal(got.view(np.uint32), deq.view(np.uint32))
    # the f16 values the GEMM stages in shared memory: RNE(d*q)
    got16 = rb.q8_0_dequant(wid, "f16").cpu().numpy()
    assert np.array_equal(got16.view(np.uint16), orc.f32_to_f16_bits(deq))
    # device encoder (rb_pack_f32_q8_0) == reference encoder, bit for bit
    wid2 = rb.pack_q8_0(w)
    got2 = rb.q8_0_dequant(wid2, "f32").cpu().numpy()
    assert np.array_equal(got2.view(np.uint32), deq.view(np.uint32))
    torch.cuda.synchronize()
    rb.check_device_errors()


# ------------------------------------------------------------------ Q8_0 GEMM
def _q8_gemm_case(rb, orc, m, n, k, seed, x_dtype="f32"):
    import torch
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w, codes, scales = q8_weight(orc, n, k, seed + 1)
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), n, k)
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[x_dtype]
    x = torch.from_numpy(a).to("cuda", tdt)
    y = rb.matmul(x, wid, out_dtype=torch.float32)
    torch.cuda.synchronize()
    rb.check_device_errors()
    got = y.cpu().numpy()
    deq = orc.q8_0_dequant(codes, scales)
    ref = orc.gemm_f64acc(a, deq)  # the reference f32 path
    return got, ref, a, deq


def test_q8_0_gemm_config1_parity(rb, orc):
    """BASELINE config #1: [512, 1024] x Q8_0 [3072, 1024]^T -> f32 [512, 3072]."""
    got, ref, a, deq = _q8_gemm_case(rb, orc, 512, 3072, 1024, seed=11)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL
    # tighter: same f16-rounded operands, only the accumulation order differs
    a16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(a))
    w16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(deq))
    ref16 = orc.gemm_f64acc(a16, w16)
    assert max_rel(got, ref16) <= 1e-5


# (1000, 1000, 512): 96-column CTA-pair tiles, one per pair, a 40-column last
# tile; (2560, 1920, 512): 96-column pair tiles, three per pair (both
# accumulator buffers in turn).
@pytest.mark.parametrize("m,n,k", [(1, 32, 32), (3, 96, 96), (129, 200, 1024), (300, 3072, 64),
                                   (77, 136, 160), (1000, 1024, 1024), (128, 6144, 1024),
                                   (1000, 1000, 512), (2560, 1920, 512)])
def test_q8_0_gemm_ragged_shapes(rb, orc, m, n, k):
    got, ref, _, _ = _q8_gemm_case(rb, orc, m, n, k, seed=m + n + k)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL


@pytest.mark.parametrize("x_dtype", ["f16", "bf16"])
def test_q8_0_gemm_half_inputs(rb, orc, x_dtype):
    got, ref, _, _ = _q8_gemm_case(rb, orc, 256, 512, 512, seed=5, x_dtype=x_dtype)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL


def test_q8_0_gemm_host_entry_matches_device(rb, orc):
    import torch
    rng = np.random.default_rng(21)
    a = rng.standard_normal((64, 256)).astype(np.float32)
    w, codes, scales = q8_weight(orc, 128, 256, 22)
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), 128, 256)
    y_host = rb.matmul_host(a, wid)
    y_dev = rb.matmul(torch.from_numpy(a).cuda(), wid).cpu().numpy()
    assert np.array_equal(y_host, y_dev)


@pytest.mark.parametrize("m", [512, 1100, 2394])
def test_host_entry_pipelined_rows(rb, orc, m):
    """Calls of rb_matmul_host with m >= 512 run in overlapped row chunks
    (copy in, matmul, copy out); Q8_0 and W8A8 results equal the device entry
    on the same inputs (W8A8 bit for bit; Q8_0 within f32 rounding)."""
    import torch
    rng = np.random.default_rng(m)
    a = rng.standard_normal((m, 1152)).astype(np.float32)
    w, codes, scales = q8_weight(orc, 640, 1152, m + 1)
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), 640, 1152)
    y_host = rb.matmul_host(a, wid)
    y_dev = rb.matmul(torch.from_numpy(a).cuda(), wid).cpu().numpy()
    assert max_rel(y_host, y_dev) <= 1e-5
    wq = rb.pack_w8a8_float(torch.from_numpy((rng.standard_normal((640, 1152)) * 0.02).astype(np.float32)).cuda())
    y_host = rb.matmul_host(a, wq)
    y_dev = rb.matmul(torch.from_numpy(a).cuda(), wq).cpu().numpy()
    assert np.array_equal(y_host, y_dev)


def test_q8_0_gemm_rejects_bad_k(rb, orc):
    import torch
    w, codes, scales = q8_weight(orc, 32, 64, 1)
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), 32, 64)
    with pytest.raises(rb.OpFailure) as ei:
        rb.matmul(torch.zeros(4, 96, device="cuda"), wid)
    assert ei.value.error.rc == -1


# ------------------------------------------------------------------ W8A8
def _w8a8_case(rb, orc, m, n, k, seed, in_scale=0.0, out_scale=0.0):
    import torch
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, ws = orc.quantize_weight_per_channel(w)
    wid = rb.pack_qat(codes, ws, n, k, in_scale, out_scale)
    xd = torch.from_numpy(x).cuda()
    return x, codes, ws, wid, xd


@pytest.mark.parametrize("m,n,k", [(1, 32, 32), (7, 100, 64), (300, 3456, 1152), (2394, 1152, 1152),
                                   (257, 1152, 4304), (129, 4304, 1152)])
def test_w8a8_bit_exact(rb, orc, m, n, k):
    import torch
    x, codes, ws, wid, xd = _w8a8_case(rb, orc, m, n, k, seed=m * 3 + n + k)
    # per-row activation quantiser (ext.rs:1263-1279)
    qd, sd = rb.quantize_rows_i8(xd)
    q, s = orc.quantize_rows_i8(x)
    assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(sd.cpu().numpy().view(np.uint32), s.view(np.uint32))
    # exact int32 accumulators
    acc = rb.matmul_i8_acc(qd, wid).cpu().numpy()
    assert np.array_equal(acc, orc.gemm_i8(q, codes))
    # full op, f32 epilogue bit for bit
    y = rb.matmul(xd, wid).cpu().numpy()
    want = orc.w8a8_matmul(x, codes, ws)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    torch.cuda.synchronize()
    rb.check_device_errors()


def test_w8a8_static_scales(rb, orc):
    """pack_qat with calibrated in/out scales (ext.rs:1256-1262, 1356-1360)."""
    x, codes, ws, wid, xd = _w8a8_case(rb, orc, 64, 96, 128, seed=9, in_scale=0.03, out_scale=0.05)
    y = rb.matmul(xd, wid).cpu().numpy()
    want = orc.w8a8_matmul(x, codes, ws, 0.03, 0.05)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


def test_w8a8_f16_output(rb, orc):
    import torch
    x, codes, ws, wid, xd = _w8a8_case(rb, orc, 50, 160, 256, seed=10)
    y = rb.matmul(xd, wid, out_dtype=torch.float16).cpu().numpy()
    want = orc.w8a8_matmul(x, codes, ws)
    assert np.array_equal(y.view(np.uint16), orc.f32_to_f16_bits(want))


# ------------------------------------------------------------------ tile policies
@pytest.fixture
def tile_policy(rb):
    """Restores the automatic GEMM tile policy after the test."""
    yield rb.set_tile_policy
    rb.set_tile_policy("auto")


@pytest.mark.parametrize("policy", ["single", "pair"])
@pytest.mark.parametrize("m,n,k", [(1, 32, 32), (300, 3456, 1152), (257, 1152, 4304), (600, 1000, 256),
                                   (1100, 4304, 1152)])
def test_w8a8_bit_exact_each_tile_policy(rb, orc, tile_policy, policy, m, n, k):
    """Single-CTA and CTA-pair (cta_group::2, 256-row) tiles both reproduce
    matmul_qat bit for bit, including M and N tails of the 256-row pair tile."""
    tile_policy(policy)
    x, codes, ws, wid, xd = _w8a8_case(rb, orc, m, n, k, seed=m + 2 * n + k)
    qd, _ = rb.quantize_rows_i8(xd)
    acc = rb.matmul_i8_acc(qd, wid).cpu().numpy()
    assert np.array_equal(acc, orc.gemm_i8(qd.cpu().numpy(), codes))
    y = rb.matmul(xd, wid).cpu().numpy()
    want = orc.w8a8_matmul(x, codes, ws)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    rb.check_device_errors()


@pytest.mark.parametrize("policy", ["single", "pair"])
@pytest.mark.parametrize("m,n,k", [(1, 32, 32), (300, 3072, 64), (1000, 1024, 1024), (600, 6144, 1024),
                                   (513, 136, 160)])
def test_q8_0_gemm_each_tile_policy(rb, orc, tile_policy, policy, m, n, k):
    tile_policy(policy)
    got, ref, a, deq = _q8_gemm_case(rb, orc, m, n, k, seed=3 * m + n + k)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL
    a16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(a))
    w16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(deq))
    assert max_rel(got, orc.gemm_f64acc(a16, w16)) <= 1e-5


@pytest.mark.parametrize("policy", ["auto", "pair"])
@pytest.mark.parametrize("m,n,k", [(512, 3072, 1024), (300, 1000, 256), (600, 6144, 1024), (5000, 1024, 512)])
def test_q8_0_gemm_f16_out_is_rounded_f32_out(rb, orc, tile_policy, policy, m, n, k):
    """The f16 output is the f32 result rounded once (same accumulators),
    including single-tile pair launches, whose dequant warps help the
    epilogue warps drain the accumulator (and a multi-tile shape, where they
    do not)."""
    import torch
    tile_policy(policy)
    rng = np.random.default_rng(m + 2 * n + 3 * k)
    w, codes, scales = q8_weight(orc, n, k, seed=m + k)
    wid = rb.pack_q8_0_blocks(orc.q8_0_to_blocks(codes, scales), n, k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to("cuda", torch.float16)
    y32 = rb.matmul(x, wid, out_dtype=torch.float32)
    y16 = rb.matmul(x, wid, out_dtype=torch.float16)
    torch.cuda.synchronize()
    rb.check_device_errors()
    assert torch.equal(y16.view(torch.int16), y32.half().view(torch.int16))
    ref = orc.gemm_f64acc(x.float().cpu().numpy(), orc.q8_0_dequant(codes, scales))
    assert cosine(y32.cpu().numpy(), ref) >= COS_MIN


def test_tile_policy_rejects_unknown(rb):
    import burn_rocket_b200._lib as L
    assert L.load().rb_set_tile_policy(7) != 0
    assert rb.set_tile_policy("auto") == "auto"


# ------------------------------------------------------------------ group-wise int8 (a7)
@pytest.mark.parametrize("m,n,k,group", [(1, 32, 32, 32), (50, 96, 256, 32), (300, 1024, 1024, 128),
                                         (129, 3072, 1024, 64), (257, 200, 384, 128), (70, 130, 1024, 512),
                                         (2394, 4304, 1152, 128), (1000, 1152, 4096, 32),
                                         (100, 200, 4096, 2048)])
def test_group_int8_matmul_bit_exact(rb, orc, m, n, k, group):
    """rocket_pack_i8 + matmul_i8 (ext.rs:939-1029, 1505-1554): codes and group
    scales of both operands, and the f32 sum of promoted int32 group partials,
    bit for bit against the oracle (host.rs:77-90, int8.rs:641-672)."""
    import torch
    rng = np.random.default_rng(m + n + k + group)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wid = rb.pack_i8(w, group)
    xd = torch.from_numpy(x).cuda()
    qd, sd = rb.quantize_row_groups(xd, group)
    q, s = orc.quantize_rows_groups(x, group)
    assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(sd.cpu().numpy().view(np.uint32), s.view(np.uint32))
    y = rb.matmul(xd, wid).cpu().numpy()
    wq, ws = orc.quantize_rows_groups(w, group)
    want = orc.matmul_gw(q, s, wq, ws, group)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    # and close to the float product (the reference's host.rs:224-275 bound)
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    assert np.abs(y - ref).max() <= 0.1 * max(np.abs(ref).max(), 1.0)
    # f16 activations are quantised as given (their own codes); f16 output = RNE of the f32 sum
    y16 = rb.matmul(xd.half(), wid, out_dtype=torch.float16).cpu().numpy()
    q16, s16 = orc.quantize_rows_groups(x.astype(np.float16).astype(np.float32), group)
    want16 = orc.matmul_gw(q16, s16, wq, ws, group)
    assert np.array_equal(y16.view(np.uint16), orc.f32_to_f16_bits(want16))
    rb.check_device_errors()


def test_group_int8_rejects_bad_group(rb):
    import burn_rocket_b200 as rbm
    with pytest.raises(rbm.OpFailure):
        rb.pack_i8(np.zeros((32, 96), np.float32), 64)   # 64 does not divide 96
    with pytest.raises(rbm.OpFailure):
        rb.pack_i8(np.zeros((32, 96), np.float32), 48)   # not a multiple of 32


# ------------------------------------------------------------------ fp16-resident weights (a3-a5)
@pytest.mark.parametrize("m,n,k", [(1, 32, 32), (77, 136, 160), (512, 3072, 1024), (2000, 1024, 2048)])
def test_f16_weight_matmul(rb, orc, m, n, k):
    """rocket_pack keeps the weight as f16 (ext.rs:829-850): f16 x f16 products
    with f32 accumulation; only the summation order differs from the f64
    product of the same f16 operands."""
    import torch
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wid = rb.pack(w)
    for x_dt in (torch.float32, torch.float16):
        y = rb.matmul(torch.from_numpy(a).cuda().to(x_dt), wid, out_dtype=torch.float32).cpu().numpy()
        a16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(a))
        w16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(w))
        assert max_rel(y, orc.gemm_f64acc(a16, w16)) <= 1e-5
    rb.check_device_errors()


def test_f16_pack2_pack3_concatenate_and_policies(rb, orc, tile_policy):
    import torch
    rng = np.random.default_rng(3)
    k = 256
    parts = [(rng.standard_normal((n, k)) * 0.02).astype(np.float32) for n in (64, 96, 32)]
    x = torch.from_numpy(rng.standard_normal((300, k)).astype(np.float32)).cuda()
    full = rb.matmul(x, rb.pack(np.concatenate(parts, 0))).cpu().numpy()
    for policy in ("single", "pair"):
        tile_policy(policy)
        y3 = rb.matmul(x, rb.pack3(*parts)).cpu().numpy()
        assert np.array_equal(y3, full) or max_rel(y3, full) <= 1e-6
    y2 = rb.matmul(x, rb.pack2(parts[0], parts[1])).cpu().numpy()
    assert max_rel(y2, full[:, :160]) <= 1e-6
    # bf16 host weights are rounded to f16 like the reference's pack
    wb = torch.from_numpy(parts[0]).to(torch.bfloat16)
    yb = rb.matmul(x, rb.pack(wb)).cpu().numpy()
    wb16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(wb.float().numpy()))
    a16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(x.cpu().numpy()))
    assert max_rel(yb, orc.gemm_f64acc(a16, wb16)) <= 1e-5


# ------------------------------------------------------------------ gated (SwiGLU) epilogue

@pytest.mark.parametrize("policy", ["auto", "single", "pair"])
@pytest.mark.parametrize("m,inter,k", [(1, 64, 64), (300, 768, 1024), (1000, 3072, 1024), (4096, 192, 256)])
def test_gated_q8_0_matmul_is_silu_mul_of_gate_up(rb, orc, tile_policy, policy, m, inter, k):
    """pack_gated_q8_0(gate, up) then matmul == silu(x gate^T) * (x up^T) of the
    Q8_0-dequantised weights (host.rs:31-38), f16 output; cosine / max-rel bar."""
    import torch
    tile_policy(policy)
    rng = np.random.default_rng(m + inter + k)
    gate = (rng.standard_normal((inter, k)) * 0.02).astype(np.float32)
    up = (rng.standard_normal((inter, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    wid = rb.pack_gated_q8_0(torch.from_numpy(gate), torch.from_numpy(up))
    assert rb.weight_info(wid)[1] == inter
    xd = torch.from_numpy(x).cuda().half()
    y = torch.empty(m, inter, dtype=torch.float16, device="cuda")
    rb.matmul(xd, wid, out=y)
    torch.cuda.synchronize()
    rb.check_device_errors()
    x16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(x)).astype(np.float64)
    gd = orc.q8_0_dequant(*orc.q8_0_quantize(gate)).astype(np.float64)
    ud = orc.q8_0_dequant(*orc.q8_0_quantize(up)).astype(np.float64)
    g, u = x16 @ gd.T, x16 @ ud.T
    ref = g / (1.0 + np.exp(-g)) * u
    got = y.float().cpu().numpy()
    assert cosine(got, ref) >= COS_MIN, cosine(got, ref)
    assert max_rel(got, ref) <= MAX_REL, max_rel(got, ref)


def test_gated_pack_contract(rb):
    import torch
    with pytest.raises(Exception):
        rb.pack_gated_q8_0(torch.zeros(96, 64), torch.zeros(96, 64))  # rows not a multiple of 64
    wid = rb.pack_gated_q8_0(torch.zeros(64, 64), torch.zeros(64, 64))
    with pytest.raises(Exception):  # the fused output is f16 only
        rb.matmul(torch.zeros(4, 64, device="cuda"), wid, out=torch.empty(4, 64, device="cuda"))


# ------------------------------------------------------------------ fused activation (GELU-tanh)

def _gelu_tanh(v):
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


@pytest.mark.parametrize("policy", ["auto", "single", "pair"])
@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (300, 4304, 1152), (2394, 1000, 256)])
def test_w8a8_fused_gelu(rb, orc, tile_policy, policy, m, n, k):
    """set_weight_activation(w, "gelu_tanh"): matmul == gelu_tanh(the W8A8
    product) (host.rs:15-18) with f16 output."""
    import torch
    tile_policy(policy)
    x, codes, ws, wid, xd = _w8a8_case(rb, orc, m, n, k, seed=m + n + 7 * k)
    rb.set_weight_activation(wid, "gelu_tanh")
    y = torch.empty(m, n, dtype=torch.float16, device="cuda")
    rb.matmul(xd, wid, out=y)
    torch.cuda.synchronize()
    rb.check_device_errors()
    ref = _gelu_tanh(orc.w8a8_matmul(x, codes, ws).astype(np.float64))
    got = y.float().cpu().numpy()
    assert cosine(got, ref) >= COS_MIN, cosine(got, ref)
    assert max_rel(got, ref) <= MAX_REL, max_rel(got, ref)
    rb.set_weight_activation(wid, "none")
    with pytest.raises(ValueError):
        rb.set_weight_activation(wid, "relu")


def test_q8_0_fused_gelu_and_contract(rb, orc):
    import torch
    m, n, k = 200, 512, 256
    w, codes, scales = q8_weight(orc, n, k, seed=5)
    wid = rb.pack_q8_0(torch.from_numpy(w))
    rb.set_weight_activation(wid, "gelu_tanh")
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    y = torch.empty(m, n, dtype=torch.float16, device="cuda")
    rb.matmul(torch.from_numpy(x).cuda().half(), wid, out=y)
    torch.cuda.synchronize()
    x16 = orc.f16_bits_to_f32(orc.f32_to_f16_bits(x)).astype(np.float64)
    ref = _gelu_tanh(x16 @ orc.q8_0_dequant(codes, scales).astype(np.float64).T)
    got = y.float().cpu().numpy()
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL
    with pytest.raises(Exception):  # fused activations write f16 only
        rb.matmul(torch.from_numpy(x).cuda(), wid, out=torch.empty(m, n, device="cuda"))
    rb.check_device_errors()
