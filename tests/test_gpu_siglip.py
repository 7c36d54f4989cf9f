"""Device parity of the SigLIP-style W8A8 tower (BASELINE config #4) and the
kernels it adds — LayerNorm, GELU-tanh, the device per-channel int8 weight
quantiser, head_dim 72 attention — against the CPU oracle.

Integer work (weight codes, the W8A8 matmul) is compared bit for bit; float
glue against f64 formulas; the 2-layer tower against oracle/siglip_ref.py on
the same seeded weights at the real widths (cosine >= 0.9999 per image,
max |err| <= 1e-2 * max |ref|).
"""
import math
from dataclasses import replace

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def max_rel(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / (np.abs(want).max() + 1e-30))


@pytest.mark.parametrize("d", [1152, 768])
def test_add_layer_norm(rb, d):
    import torch
    import burn_rocket_b200._lib as L
    from oracle.siglip_ref import layer_norm
    lib = L.load()
    rng = np.random.default_rng(d)
    rows = 77
    x = (rng.standard_normal((rows, d)) * 3 + 1).astype(np.float32)
    delta = rng.standard_normal((rows, d)).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    dd = torch.from_numpy(delta).cuda()
    gd, bd = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
    h = torch.empty(rows, d, dtype=torch.float16, device="cuda")
    assert lib.rb_add_layer_norm(xd.data_ptr(), None, gd.data_ptr(), bd.data_ptr(), 1e-6, h.data_ptr(), rows, d,
                                 None) == 0, L.last_error()
    want = layer_norm(x.astype(np.float64), g, b, 1e-6)
    np.testing.assert_allclose(h.float().cpu().numpy(), want, rtol=2e-3, atol=2e-3)
    assert lib.rb_add_layer_norm(xd.data_ptr(), dd.data_ptr(), gd.data_ptr(), bd.data_ptr(), 1e-6, h.data_ptr(),
                                 rows, d, None) == 0, L.last_error()
    x2 = x.astype(np.float64) + delta.astype(np.float64)
    np.testing.assert_allclose(xd.cpu().numpy(), x2, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(h.float().cpu().numpy(), layer_norm(x2, g, b, 1e-6), rtol=2e-3, atol=2e-3)
    assert lib.rb_add_layer_norm(xd.data_ptr(), None, gd.data_ptr(), bd.data_ptr(), 1e-6, h.data_ptr(), rows, 1000,
                                 None) != 0
    rb.check_device_errors()


@pytest.mark.parametrize("d", [768, 1024, 1152])
def test_add_layer_norm_quant_matches_layer_norm_then_quantiser(rb, d):
    """The fused LayerNorm + W8A8 row quantiser gives the codes and scales of
    rb_add_layer_norm followed by rb_quantize_rows_i8, bit for bit, and the
    code-input W8A8 matmul equals rb_matmul on the f16 rows bit for bit."""
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    rows = 333
    g = torch.Generator(device="cuda").manual_seed(d)
    x0 = torch.randn(rows, d, device="cuda", generator=g) * 3
    delta = (torch.randn(rows, d, device="cuda", generator=g)).half()
    gw = 1.0 + 0.1 * torch.randn(d, device="cuda", generator=g)
    bw = 0.1 * torch.randn(d, device="cuda", generator=g)
    xa, xb = x0.clone(), x0.clone()
    h = torch.empty(rows, d, dtype=torch.float16, device="cuda")
    assert lib.rb_add_layer_norm(xa.data_ptr(), delta.data_ptr(), gw.data_ptr(), bw.data_ptr(), 1e-6, h.data_ptr(),
                                 rows, d, None) == 0
    codes = torch.empty(rows, d, dtype=torch.int8, device="cuda")
    scales = torch.empty(rows, dtype=torch.float32, device="cuda")
    assert lib.rb_add_layer_norm_quant(xb.data_ptr(), delta.data_ptr(), gw.data_ptr(), bw.data_ptr(), 1e-6,
                                       codes.data_ptr(), scales.data_ptr(), rows, d, None) == 0
    torch.cuda.synchronize()
    assert torch.equal(xa, xb)  # the residual stream is updated alike
    q, s = rb.quantize_rows_i8(h)
    assert torch.equal(codes, q)
    assert torch.equal(scales.view(torch.int32), s.view(torch.int32))
    rng = np.random.default_rng(d)
    n = 256
    wid = rb.pack_qat(rng.integers(-127, 128, size=(n, d), dtype=np.int8), rng.random(n).astype(np.float32) * 1e-3,
                      n, d)
    y1 = torch.empty(rows, n, dtype=torch.float16, device="cuda")
    y2 = torch.empty_like(y1)
    rb.matmul(h, wid, out=y1)
    assert lib.rb_matmul_w8a8_codes(wid.id, codes.data_ptr(), scales.data_ptr(), rows, d, y2.data_ptr(),
                                    L.DTYPE_F16, None) == 0
    torch.cuda.synchronize()
    rb.check_device_errors()
    assert torch.equal(y1, y2)


def test_gelu_in_place(rb):
    import torch
    import burn_rocket_b200._lib as L
    from oracle.siglip_ref import gelu_tanh
    lib = L.load()
    rng = np.random.default_rng(4)
    y = (rng.standard_normal(4304 * 9) * 3).astype(np.float16)
    yd = torch.from_numpy(y).cuda()
    assert lib.rb_gelu(yd.data_ptr(), y.size, None) == 0, L.last_error()
    want = gelu_tanh(y.astype(np.float64))
    np.testing.assert_allclose(yd.float().cpu().numpy(), want, rtol=2e-3, atol=2e-3)
    assert lib.rb_gelu(yd.data_ptr(), 12, None) != 0  # count % 8


@pytest.mark.parametrize("n,k", [(3456, 1152), (1152, 4304), (100, 48)])
def test_device_weight_quantiser_matches_pack_qat(rb, orc, n, k):
    """rb_pack_f32_w8a8_device == pack_qat of the oracle's per-channel codes:
    the two weights give bit-identical int32 accumulators and f32 outputs."""
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16).astype(np.float32)
    w[0, :] = 0.0  # an all-zero channel takes the 1e-12 scale floor
    wd = torch.from_numpy(w).cuda()
    wid_dev = lib.rb_pack_f32_w8a8_device(wd.data_ptr(), n, k, 0.0, 0.0)
    assert wid_dev > 0, L.last_error()
    codes, ws = orc.quantize_weight_per_channel(w)
    wid_ref = rb.pack_qat(codes, ws, n, k)
    x = rng.standard_normal((67, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y_dev = rb.matmul(xd, rb.WeightId(int(wid_dev))).cpu().numpy()
    y_ref = rb.matmul(xd, wid_ref).cpu().numpy()
    assert np.array_equal(y_dev.view(np.uint32), y_ref.view(np.uint32))
    want = orc.w8a8_matmul(x, codes, ws)
    assert np.array_equal(y_dev.view(np.uint32), want.view(np.uint32))
    qd, _ = rb.quantize_rows_i8(xd)
    acc = rb.matmul_i8_acc(qd, rb.WeightId(int(wid_dev))).cpu().numpy()
    assert np.array_equal(acc, orc.gemm_i8(qd.cpu().numpy(), codes))
    rb.check_device_errors()


def test_batched_head_dim_72_matches_oracle(rb, orc):
    """16 heads x 72 over back-to-back images read from a fused q|k|v buffer
    (the tower's layout) against the oracle, image by image."""
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    B, S, H, D = 3, 211, 16, 72
    hq = H * D
    ld = 3 * hq
    rng = np.random.default_rng(72)
    qkv = orc.f32_to_f16_bits(rng.standard_normal((B * S, ld)).astype(np.float32))
    qd = torch.from_numpy(qkv.view(np.float16)).cuda()
    out = torch.empty(B * S, hq, dtype=torch.float16, device="cuda")
    p = qd.data_ptr()
    rc = lib.rb_attention_batched(p, ld, p + hq * 2, ld, p + 2 * hq * 2, ld, out.data_ptr(), hq, L.DTYPE_F16,
                                  B, S, S, H, H, D, 1 / math.sqrt(D), 0.0, L.MASK_NONE, -1, 0, 0, None)
    assert rc == 0, L.last_error()
    got = out.float().cpu().numpy()
    rb.check_device_errors()
    for b in range(B):
        rows = slice(b * S, (b + 1) * S)
        q = np.ascontiguousarray(qkv[rows, :hq])
        k = np.ascontiguousarray(qkv[rows, hq:2 * hq])
        v = np.ascontiguousarray(qkv[rows, 2 * hq:])
        ref = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, H, H, D, 1 / math.sqrt(D)))
        assert cosine(got[rows], ref) >= 0.9999, (b, cosine(got[rows], ref))
        assert max_rel(got[rows], ref) <= 1e-2


def test_siglip_forward_matches_oracle(rb):
    import torch
    from burn_rocket_b200.siglip import SiglipConfig, SiglipTower
    from oracle import siglip_ref
    cfg = replace(SiglipConfig(), layers=2, patches=197)
    images = 2
    hw = siglip_ref.make_host_weights(cfg, seed=11)
    tower = SiglipTower(cfg, images, host_weights=hw)
    rng = np.random.default_rng(12)
    x = rng.standard_normal((images * cfg.patches, cfg.hidden)).astype(np.float32)
    tower.patches.copy_(torch.from_numpy(x))
    got = tower.forward_device().float().cpu().numpy()
    rb.check_device_errors()
    want = siglip_ref.forward(hw, cfg, x, images)
    for im in range(images):
        rows = slice(im * cfg.patches, (im + 1) * cfg.patches)
        assert cosine(got[rows], want[rows]) >= 0.9999, (im, cosine(got[rows], want[rows]))
    assert max_rel(got, want) <= 1e-2, max_rel(got, want)


def test_siglip_graph_replay_equals_eager(rb):
    import torch
    from burn_rocket_b200.siglip import SiglipConfig, SiglipTower
    cfg = replace(SiglipConfig(), layers=2, patches=300)
    tower = SiglipTower(cfg, 2, seed=3)
    tower.patches.copy_(torch.randn(tower.T, cfg.hidden, device="cuda"))
    eager = tower.forward_device().clone()
    tower.capture()
    tower.patches.mul_(1.0)
    replay = tower.run().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, replay)
    out = tower.encode_host(tower.patches.cpu().pin_memory())
    assert torch.equal(out, eager.cpu())
    rb.check_device_errors()


def test_siglip_encode_host_overlapped_halves(rb):
    """encode_host(overlap=True) runs the images in two halves from their own
    graphs, overlapping the copies with the other half's compute; twice in a
    row, it matches the whole-batch forward (up to attention's f32 summation
    order)."""
    import torch
    from burn_rocket_b200.siglip import SiglipConfig, SiglipTower
    cfg = replace(SiglipConfig(), layers=2, patches=300)
    tower = SiglipTower(cfg, 5, seed=4)
    tower.patches.copy_(torch.randn(tower.T, cfg.hidden, device="cuda"))
    ref = tower.forward_device().float().cpu()
    hp = tower.patches.cpu().pin_memory()
    for _ in range(2):
        out = tower.encode_host(hp, overlap=True).float()
        cos = torch.nn.functional.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
        assert cos >= 0.9999, cos
        assert (out - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    rb.check_device_errors()
