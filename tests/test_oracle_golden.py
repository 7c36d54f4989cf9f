"""Pins the CPU oracle to the reference's own known-answer tests.

Each test restates a reference test (file:line) on the oracle: if the oracle
drifts from burn-rocket's arithmetic, these fail before any device test runs.
CPU only.
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc

INF = float("inf")


def xorshift_unit(seed):
    """rand_unit of crates/burn-rocket/src/host.rs:180-186: xorshift64, [-1, 1)."""
    mask = (1 << 64) - 1
    s = seed
    while True:
        s ^= (s << 13) & mask
        s ^= s >> 7
        s ^= (s << 17) & mask
        yield np.float32(np.float32(s >> 40) / np.float32(1 << 23)) - np.float32(1.0)


def xorshift_f16(seed):
    """rnd of crates/rocket-npu/src/attn/oneshot.rs:668-673: f16 in [-0.5, 0.5)."""
    mask = (1 << 64) - 1
    s = seed
    while True:
        s ^= (s << 13) & mask
        s ^= s >> 7
        s ^= (s << 17) & mask
        v = np.float32(np.float32(s >> 40) / np.float32(1 << 24)) - np.float32(0.5)
        yield int(orc.f32_to_f16_bits(np.array([v], np.float32))[0])


# ------------------------------------------------------------------ f16 codec
def test_f32_to_f16_matches_ieee_rne():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0,
        rng.standard_normal(20000).astype(np.float32) * 1e-5,   # f16 subnormals
        rng.standard_normal(20000).astype(np.float32) * 6e4,    # overflow edge
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, -65520.0, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, np.inf, -np.inf], np.float32),
    ])
    got = orc.f32_to_f16_bits(x)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    back = orc.f16_bits_to_f32(got)
    assert np.array_equal(back, want.view(np.float16).astype(np.float32))


def test_f64_to_f16_is_single_rounding():
    # values straddling f16 ties: a single rounding from f64 must win over
    # the f64 -> f32 -> f16 double rounding (ops/mod.rs:123-133).
    rng = np.random.default_rng(2)
    vals = list(rng.standard_normal(5000) * 3.0) + [1.0 + 2.0 ** -11 + 2.0 ** -40,
                                                   -(1.0 + 2.0 ** -11 + 2.0 ** -40), 1.0 + 2.0 ** -11,
                                                   65519.0, 65520.0, 6.0e-8, 2.0 ** -24 * 0.5]
    for v in vals:
        want = int(np.array([v], np.float64).astype(np.float16).view(np.uint16)[0])
        assert orc.f64_to_f16_bits(v) == want, v


# ------------------------------------------------------------------ Q8_0 codec
def test_q8_0_block_dequant_kat():
    """src/util/gguf.rs:250-260: one block, scale 0.5, q = [-1, 0, 1, 0...]."""
    raw = np.zeros(34, np.uint8)
    raw[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    raw[2] = 0xFF
    raw[3] = 0x00
    raw[4] = 0x01
    v = orc.q8_0_dequant_blocks(raw)
    assert v[0] == -0.5 and v[1] == 0.0 and v[2] == 0.5
    assert np.all(v[3:] == 0.0)


def test_q8_0_encoder_properties():
    """q8_bench.rs:199-219: d = f16(amax/127), codes against the stored scale."""
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[5, 40] = 1.75  # outlier block
    codes, scales = orc.q8_0_quantize(w)
    d = orc.f16_bits_to_f32(scales)
    blk = w.reshape(64, 8, 32)
    amax = np.abs(blk).max(-1)
    assert np.array_equal(scales, (amax / np.float32(127.0)).astype(np.float32).astype(np.float16).view(np.uint16))
    cb = codes.reshape(64, 8, 32)
    # the block max lands on +-127 (up to the scale's f16 rounding: 126 or 127)
    imax = np.abs(blk).argmax(-1)
    top = np.take_along_axis(np.abs(cb.astype(np.int32)), imax[..., None], -1)[..., 0]
    assert np.all(top >= 126)
    assert np.abs(codes).max() <= 127
    deq = orc.q8_0_dequant(codes, scales)
    err = np.abs(deq - w).reshape(64, 8, 32).max(-1)
    assert np.all(err <= d * 0.5 * (1 + 1e-6) + 1e-12)
    # planar and GGUF-block decodes agree bit for bit
    blocks = orc.q8_0_to_blocks(codes, scales)
    assert np.array_equal(orc.q8_0_dequant_blocks(blocks).reshape(64, 256), deq)
    # rounding is half away from zero (Rust f32::round): an exact .5 tie
    wt = np.zeros((1, 32), np.float32)
    wt[0, 0] = 127.0
    wt[0, 1] = 2.5
    wt[0, 2] = -2.5
    c, s = orc.q8_0_quantize(wt)
    assert orc.f16_bits_to_f32(s)[0, 0] == 1.0
    assert c[0, 1] == 3 and c[0, 2] == -3


def test_q8_0_zero_block_stays_zero():
    codes, scales = orc.q8_0_quantize(np.zeros((2, 64), np.float32))
    assert np.all(codes == 0) and np.all(scales == 0)


# ------------------------------------------------------------------ int8 quantisers
def test_static_code_ties_to_even_and_saturates():
    """ext.rs:2256-2272 (static_codes_round_half_to_even_and_saturate)."""
    assert orc.static_code(0.5, 1.0) == 0
    assert orc.static_code(1.5, 1.0) == 2
    assert orc.static_code(2.5, 1.0) == 2
    assert orc.static_code(-0.5, 1.0) == 0
    assert orc.static_code(-1.5, 1.0) == -2
    assert orc.static_code(1000.0, 1.0) == 127
    assert orc.static_code(-1000.0, 1.0) == -128
    scale = np.float32(0.0173)
    inv = np.float32(1.0) / scale
    for c in [-128, -77, -1, 0, 3, 64, 127]:
        assert orc.static_code(np.float32(c) * scale, inv) == c


def test_dynamic_row_quantiser():
    """matmul_qat with in_scale == 0 (ext.rs:1263-1279)."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((7, 96)).astype(np.float32)
    x[3] = 0.0
    q, s = orc.quantize_rows_i8(x)
    amax = np.abs(x).max(1)
    want_s = np.maximum(amax / np.float32(127.0), np.float32(1e-12)).astype(np.float32)
    assert np.array_equal(s, want_s)
    inv = (np.float32(1.0) / want_s).astype(np.float32)
    want_q = np.clip(np.rint(x * inv[:, None]), -128, 127).astype(np.int8)
    assert np.array_equal(q, want_q)
    assert np.all(q[3] == 0) and s[3] == np.float32(1e-12)


def test_int8_group_roundtrip_error_bound():
    """host.rs:188-222 (int8_quantize_roundtrip_error_bound)."""
    k, group = 128, 32
    gen = xorshift_unit(0x1234_5678_9ABC_DEF0)
    x = np.array([next(gen) for _ in range(k)], np.float32)
    x[70] = 9.5
    q, s = orc.quantize_row_groups(x, group)
    for g in range(k // group):
        seg = x[g * group:(g + 1) * group]
        amax = np.abs(seg).max()
        assert abs(s[g] - amax / 127.0) <= 1e-9 * max(amax, 1.0)
        deq = q[g * group:(g + 1) * group].astype(np.float32) * s[g]
        assert np.all(np.abs(seg - deq) <= s[g] * 0.5 + 1e-6)
    assert q[70] == 127
    assert s[2] > s[1]
    zq, zs = orc.quantize_row_groups(np.zeros(32, np.float32), 32)
    assert zs[0] > 0 and np.isfinite(zs[0]) and np.all(zq == 0)


def test_int8_groupwise_matmul_is_close():
    """host.rs:224-275: sum_g a_s[m,g] b_s[n,g] * partial within 10%."""
    m, k, n, group = 8, 64, 8, 32
    gen = xorshift_unit(7)
    a = np.array([next(gen) * np.float32(2.0) for _ in range(m * k)], np.float32).reshape(m, k)
    b = np.array([next(gen) for _ in range(n * k)], np.float32).reshape(n, k)
    ng = k // group
    aq = np.zeros((m, k), np.int8)
    as_ = np.zeros((m, ng), np.float32)
    bq = np.zeros((n, k), np.int8)
    bs = np.zeros((n, ng), np.float32)
    for r in range(m):
        aq[r], as_[r] = orc.quantize_row_groups(a[r], group)
    for r in range(n):
        bq[r], bs[r] = orc.quantize_row_groups(b[r], group)
    for r in range(m):
        for c in range(n):
            want = float(np.dot(a[r].astype(np.float64), b[c]))
            got = 0.0
            for g in range(ng):
                part = int(np.dot(aq[r, g * group:(g + 1) * group].astype(np.int32),
                                  bq[c, g * group:(g + 1) * group].astype(np.int32)))
                got += as_[r, g] * bs[c, g] * part
            assert abs(got - want) <= 0.1 * max(abs(want), 1.0)


def test_w8a8_epilogue_order_and_exact_int():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((5, 64)).astype(np.float32)
    w = (rng.standard_normal((16, 64)) * 0.02).astype(np.float32)
    codes, ws = orc.quantize_weight_per_channel(w)
    q, rs = orc.quantize_rows_i8(x)
    acc = orc.gemm_i8(q, codes)
    assert np.array_equal(acc, q.astype(np.int64) @ codes.astype(np.int64).T)
    y = orc.w8a8_epilogue(acc, rs, ws)
    want = acc.astype(np.float32) * (rs[:, None] * ws[None, :]).astype(np.float32)
    assert np.array_equal(y, want)
    # static output grid (out_scale != 0)
    y2 = orc.w8a8_epilogue(acc, rs, ws, 0.01)
    inv = np.float32(1.0) / np.float32(0.01)
    assert np.array_equal(y2, np.clip(np.rint(want * inv), -128, 127).astype(np.float32) * np.float32(0.01))


# ------------------------------------------------------------------ masks (masks.rs:116-300)
def keep(mode, t, j, window=-1, q0=0, k0=0):
    return orc.mask_visible(mode, window, q0, k0, t, j)


def test_causal_mask_semantics():
    for t in range(6):
        for j in range(6):
            assert keep(orc.MASK_CAUSAL, t, j) == (j <= t)


def test_window_mask_semantics():
    for t in range(8):
        for j in range(8):
            assert keep(orc.MASK_WINDOW, t, j, 3) == (abs(t - j) <= 3)


def test_causal_window_mask_semantics():
    for t in range(8):
        for j in range(8):
            assert keep(orc.MASK_CAUSAL_WINDOW, t, j, 3) == (j <= t and t - j < 3)


def test_window_mask_block_semantics_and_edges():
    n_q, n_kv, q0, k0, w = 5, 7, 10, 8, 3
    for i in range(n_q):
        for j in range(n_kv):
            assert keep(orc.MASK_WINDOW_BLOCK, i, j, w, q0, k0) == (abs((q0 + i) - (k0 + j)) <= w)
    assert keep(orc.MASK_WINDOW_BLOCK, 0, 0, 2, 0, 0)
    assert keep(orc.MASK_WINDOW_BLOCK, 0, 2, 2, 0, 0)
    assert not keep(orc.MASK_WINDOW_BLOCK, 0, 3, 2, 0, 0)
    for i in range(4):
        for j in range(5):
            assert keep(orc.MASK_WINDOW_BLOCK, i, j, 2, 20, 18) == (abs((20 + i) - (18 + j)) <= 2)


def test_causal_mask_block_semantics_offsets_and_tail():
    n_q, n_kv, q0, k0 = 4, 10, 8, 4
    for i in range(n_q):
        for j in range(n_kv):
            assert keep(orc.MASK_CAUSAL_BLOCK, i, j, -1, q0, k0) == (k0 + j <= q0 + i)
    # ragged 30k tail (masks.rs:240-262)
    n_q, n_kv, q0 = 8, 29960, 29952
    for i in range(n_q):
        for j in [0, 1, q0 + i - 1, q0 + i, min(q0 + i + 1, n_kv - 1), n_kv - 1]:
            assert keep(orc.MASK_CAUSAL_BLOCK, i, j, -1, q0, 0) == (j <= q0 + i)
    # keys wholly below / above the chunk
    assert all(keep(orc.MASK_CAUSAL_BLOCK, i, j, -1, 20, 12) for i in range(4) for j in range(8))
    assert not any(keep(orc.MASK_CAUSAL_BLOCK, i, j, -1, 20, 24) for i in range(4) for j in range(8))


def test_causal_window_block_semantics():
    n_q, n_kv, q0, k0, w = 5, 12, 16, 8, 4
    for i in range(n_q):
        for j in range(n_kv):
            q, k = q0 + i, k0 + j
            assert keep(orc.MASK_CAUSAL_BLOCK, i, j, w, q0, k0) == (k <= q and q - k < w)
    for i in range(6):
        vis = sum(keep(orc.MASK_CAUSAL_BLOCK, i, j, 2, 0, 0) for j in range(6))
        assert vis == min(i + 1, 2)


# ------------------------------------------------------------------ attention oracle
def test_fa_score_scales_caps_masks_and_clamps():
    """attn/oneshot.rs:748-761."""
    assert orc.fa_score(4.0, 0.5, 0.0, 0.0) == 2.0
    assert orc.fa_score(4.0, 0.5, 0.0, -1.0) == 1.0
    capped = orc.fa_score(60.0, 0.5, 30.0, 0.0)
    assert abs(capped - 30.0 * math.tanh(1.0)) < 1e-5 and capped < 30.0
    assert abs(orc.fa_score(1.0e4, 0.5, 30.0, 0.0) - 30.0) < 1e-4
    assert orc.fa_score(-1.0e5, 1.0, 0.0, 0.0) == -30000.0
    assert orc.fa_score(1.0, 1.0, 0.0, -INF) == -30000.0


def _tok_major(head_major, heads, n, d):
    """[heads][n][d] -> [n, heads*d]."""
    return np.ascontiguousarray(head_major.reshape(heads, n, d).transpose(1, 0, 2).reshape(n, heads * d))


def test_flash_ref_picks_the_one_visible_key():
    """attn/oneshot.rs:763-810, restated with a window-block mask that leaves
    exactly key (row+1) % kv visible... via an explicit check of the one-hot."""
    t, kv, dk, heads, hkv = 3, 5, 32, 2, 1
    gen = xorshift_f16(0x1234_5678_9ABC_DEF0)
    q = np.array([next(gen) for _ in range(heads * t * dk)], np.uint16)
    k = np.array([next(gen) for _ in range(hkv * kv * dk)], np.uint16)
    v = np.array([next(gen) for _ in range(hkv * dk * kv)], np.uint16)
    # one visible key per row: a window-block band of width 0 at offset +1
    # (query i sees key i+1 only).
    qt = _tok_major(q, heads, t, dk)
    kt = _tok_major(k, hkv, kv, dk)
    vt = _tok_major(v, hkv, kv, dk)
    out = orc.flash_attn_ref(qt, kt, vt, heads, hkv, dk, 0.125, 0.0, orc.MASK_WINDOW_BLOCK, 0, 1, 0)
    for h in range(heads):
        for row in range(t):
            j = row + 1
            assert np.array_equal(out[row, h * dk:(h + 1) * dk], vt[j, 0:dk])


def _naive(q, k, v, n_head, n_kv_heads, d, scale, softcap, vis):
    qf = orc.f16_bits_to_f32(q).astype(np.float64).reshape(-1, n_head, d)
    kf = orc.f16_bits_to_f32(k).astype(np.float64).reshape(-1, n_kv_heads, d)
    vf = orc.f16_bits_to_f32(v).astype(np.float64).reshape(-1, n_kv_heads, d)
    g = n_head // n_kv_heads
    out = np.zeros_like(qf)
    for h in range(n_head):
        s = (qf[:, h] @ kf[:, h // g].T).astype(np.float32) * np.float32(scale)
        if softcap:
            s = np.float32(softcap) * np.tanh(s / np.float32(softcap))
        s = np.where(vis, s, -np.inf).astype(np.float64)
        s = np.maximum(s, -30000.0)
        p = np.exp(s - s.max(1, keepdims=True))
        out[:, h] = (p / p.sum(1, keepdims=True)) @ vf[:, h // g]
    return out.reshape(qf.shape[0], -1)


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_flash_ref_gqa_softcap_and_no_mask_like_the_naive_reference():
    """attn/oneshot.rs:812-852 (GQA 8/2, ragged kv, softcap, mask and no mask)."""
    t, kv, dk, heads, hkv = 5, 37, 64, 8, 2
    gen = xorshift_f16(0x0BAD_C0DE_1234_5678)
    q = np.array([next(gen) for _ in range(t * heads * dk)], np.uint16).reshape(t, heads * dk)
    k = np.array([next(gen) for _ in range(kv * hkv * dk)], np.uint16).reshape(kv, hkv * dk)
    v = np.array([next(gen) for _ in range(kv * hkv * dk)], np.uint16).reshape(kv, hkv * dk)
    for softcap in [0.0, 20.0]:
        for mode, window in [(orc.MASK_CAUSAL_BLOCK, -1), (orc.MASK_NONE_BLOCK, -1)]:
            # j > i + 2 hidden == causal block with q0 = 2
            q0 = 2 if mode == orc.MASK_CAUSAL_BLOCK else 0
            vis = orc.mask_matrix(mode, t, kv, window, q0, 0)
            got = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, heads, hkv, dk, 0.125, softcap, mode, window, q0, 0))
            want = _naive(q, k, v, heads, hkv, dk, 0.125, softcap, vis)
            want16 = np.array([orc.f16_bits_to_f32(np.array([orc.f64_to_f16_bits(x)]))[0] for x in want.ravel()])
            assert cosine(got, want16) > 0.999999
            assert np.abs(got.ravel() - want16).max() < 2e-3


def test_flash_ref_emptied_row_averages_every_real_key():
    """attn/oneshot.rs:910-950."""
    t, kv, d = 1, 3, 32
    q = np.zeros((t, d), np.uint16)
    k = np.zeros((kv, d), np.uint16)
    vf = np.zeros((kv, d), np.float32)
    for c in range(d):
        vf[c % kv, c] = 3.0 * (c % kv + 1)
    v = orc.f32_to_f16_bits(vf)
    # all keys masked: a causal block whose keys lie wholly above the query
    out = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, 1, 1, d, 0.125, 0.0, orc.MASK_CAUSAL_BLOCK, -1, 0, 10))
    for c in range(d):
        assert abs(out[0, c] - (c % kv + 1)) < 1e-3


def test_tiled_cpu_attention_equals_one_pass():
    """attn/mod.rs:1902-1967: the online (tiled) fold equals one materialised pass."""
    rng = np.random.default_rng(6)
    n, h, hkv, d = 150, 4, 2, 64
    q = rng.standard_normal((n, h * d)).astype(np.float32)
    k = rng.standard_normal((n, hkv * d)).astype(np.float32)
    v = rng.standard_normal((n, hkv * d)).astype(np.float32)
    q16, k16, v16 = (orc.f32_to_f16_bits(a) for a in (q, k, v))
    qf, kf, vf = (orc.f16_bits_to_f32(a) for a in (q16, k16, v16))
    for causal in (False, True):
        tiled = orc.attention_cpu(qf, kf, vf, h, hkv, d, 0.125, causal)
        one = orc.f16_bits_to_f32(orc.flash_attn_ref(q16, k16, v16, h, hkv, d, 0.125, 0.0,
                                                     orc.MASK_CAUSAL if causal else orc.MASK_NONE))
        assert cosine(tiled, one) > 0.99999
        assert np.abs(tiled - one).max() < 2e-3
