"""Device parity of the glue kernels and of the Qwen3-Embedding forward
(BASELINE config #3 architecture) against the CPU oracle.

Glue ops compare with plain f64 formulas of crates/burn-rocket/src/host.rs;
the forward compares the L2-normalised embeddings with oracle/qwen3_ref.py on
the same seeded weights (2 layers, real widths). Tolerance (north star):
cosine >= 0.9999 and max |err| <= 1e-2 * max |ref|.
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


def test_rms_norm_and_gated_glue(rb):
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((37, 1024)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    y = torch.empty_like(xd)
    assert lib.rb_rms_norm(xd.data_ptr(), L.DTYPE_F32, wd.data_ptr(), 1e-6, y.data_ptr(), L.DTYPE_F32, 37, 1024,
                           None) == 0
    want = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * w
    torch.cuda.synchronize()
    assert np.abs(y.cpu().numpy() - want).max() < 1e-5 * np.abs(want).max()
    g = rng.standard_normal(5000).astype(np.float32) * 4
    u = rng.standard_normal(5000).astype(np.float32)
    gd, ud = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    o = torch.empty_like(gd)
    assert lib.rb_silu_mul(gd.data_ptr(), ud.data_ptr(), L.DTYPE_F32, o.data_ptr(), 5000, None) == 0
    g64 = g.astype(np.float64)
    np.testing.assert_allclose(o.cpu().numpy(), g64 / (1 + np.exp(-g64)) * u, rtol=1e-5, atol=1e-6)
    assert lib.rb_gelu_mul(gd.data_ptr(), ud.data_ptr(), L.DTYPE_F32, o.data_ptr(), 5000, None) == 0
    k = math.sqrt(2 / math.pi)
    gel = 0.5 * g64 * (1 + np.tanh(k * (g64 + 0.044715 * g64 ** 3))) * u
    np.testing.assert_allclose(o.cpu().numpy(), gel, rtol=1e-5, atol=1e-5)


def test_rope(rb):
    import torch
    import burn_rocket_b200._lib as L
    from oracle.qwen3_ref import rope_tables
    lib = L.load()
    rng = np.random.default_rng(2)
    B, S, HQ, HK, D = 2, 40, 4, 2, 128
    cos, sin = rope_tables(S, D, 1e6)
    cd, sd = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    x = rng.standard_normal((B, S, HQ, D)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    assert lib.rb_rope(xd.data_ptr(), L.DTYPE_F32, cd.data_ptr(), sd.data_ptr(), y.data_ptr(), B, S, HQ, D, None) == 0
    half = D // 2
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    want = np.concatenate([x[..., :half] * c - x[..., half:] * s, x[..., half:] * c + x[..., :half] * s], -1)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("hq,hk", [(4, 2), (16, 8), (32, 4), (36, 4)])
def test_qk_norm_rope(rb, hq, hk):
    """Per-head RMSNorm + RoPE in place on a fused q|k|v buffer against the f64
    formula, through both device forms: one warp per token with 16-byte
    accesses (row stride a multiple of 8 halves, at most 36 q+k heads) and the
    half-warp-per-head form (any other stride, more heads). The two differ
    only in the order of each head's sum of squares, so they agree within one
    f16 step; v columns and the padding columns stay untouched."""
    import torch
    import burn_rocket_b200._lib as L
    from oracle.qwen3_ref import rope_tables
    lib = L.load()
    rng = np.random.default_rng(hq * 100 + hk)
    B, S, D = 2, 40, 128
    half = D // 2
    cos, sin = rope_tables(S, D, 1e6)
    cd, sd = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    width = (hq + 2 * hk) * D
    src16 = (rng.standard_normal((B * S, width)) * 3).astype(np.float16)
    wq = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wk = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wqd, wkd = torch.from_numpy(wq).cuda(), torch.from_numpy(wk).cuda()
    src = src16.astype(np.float64).reshape(B, S, hq + 2 * hk, D)
    heads = src[:, :, :hq + hk]
    wts = np.concatenate([np.tile(wq, (hq, 1)), np.tile(wk, (hk, 1))])[None, None]
    nrm = heads / np.sqrt((heads ** 2).mean(-1, keepdims=True) + 1e-6) * wts
    rot = np.concatenate([nrm[..., :half] * c - nrm[..., half:] * s, nrm[..., half:] * c + nrm[..., :half] * s], -1)
    outs = []
    for pad in (0, 4):  # pad 0: the 16-byte form when hq + hk <= 36; pad 4: the half-warp form
        ld = width + pad
        buf = np.full((B * S, ld), 7.0, np.float16)
        buf[:, :width] = src16
        t = torch.from_numpy(buf).cuda()
        assert lib.rb_qk_norm_rope(t.data_ptr(), ld, B * S, hq, hk, D, wqd.data_ptr(), wkd.data_ptr(), 1e-6,
                                   cd.data_ptr(), sd.data_ptr(), S, None) == 0
        torch.cuda.synchronize()
        got16 = t.cpu().numpy()
        assert np.all(got16[:, width:] == 7.0)
        got = got16[:, :width].astype(np.float64).reshape(B, S, hq + 2 * hk, D)
        assert np.array_equal(got[:, :, hq + hk:], src[:, :, hq + hk:])  # v untouched
        err = np.abs(got[:, :, :hq + hk] - rot)
        # f16 output: within 1e-3 of the row's scale (two f16 steps at |x| ~ 4)
        assert err.max() < 1e-3 * np.abs(rot).max(), (pad, err.max())
        outs.append(got16[:, :width])
    a = outs[0].astype(np.float16).view(np.int16).astype(np.int64)
    b = outs[1].astype(np.float16).view(np.int16).astype(np.int64)
    assert np.abs(a - b).max() <= 1
    # a row stride that does not cover the q and k columns is rejected
    t = torch.from_numpy(src16.copy()).cuda()
    assert lib.rb_qk_norm_rope(t.data_ptr(), (hq + hk) * D - 8, B * S, hq, hk, D, wqd.data_ptr(), wkd.data_ptr(),
                               1e-6, cd.data_ptr(), sd.data_ptr(), S, None) == L.RB_E_SHAPE


def test_batched_attention_equals_per_sequence(rb):
    """rb_attention_batched over back-to-back sequences read from a fused
    q|k|v buffer equals one rb_attention call per sequence, bit for bit."""
    import torch
    import burn_rocket_b200._lib as L
    lib = L.load()
    B, S, H, KV, D = 3, 200, 4, 2, 128
    ld = (H + 2 * KV) * D
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(B * S, ld, device="cuda", generator=g).half()
    out = torch.empty(B * S, H * D, dtype=torch.float16, device="cuda")
    p = qkv.data_ptr()
    for mode in (L.MASK_NONE, L.MASK_CAUSAL):
        rc = lib.rb_attention_batched(p, ld, p + H * D * 2, ld, p + (H + KV) * D * 2, ld, out.data_ptr(), H * D,
                                      L.DTYPE_F16, B, S, S, H, KV, D, 1 / math.sqrt(D), 0.0, mode, -1, 0, 0, None)
        assert rc == 0, L.last_error()
        for b in range(B):
            rows = slice(b * S, (b + 1) * S)
            q = qkv[rows, :H * D].contiguous()
            k = qkv[rows, H * D:(H + KV) * D].contiguous()
            v = qkv[rows, (H + KV) * D:].contiguous()
            one = rb.attention(q, k, v, H, KV, D, 1 / math.sqrt(D), None, mode == L.MASK_CAUSAL)
            assert torch.equal(one, out[rows]), (mode, b)
    rb.check_device_errors()


@pytest.mark.parametrize("causal", [False, True])
def test_qwen3_forward_matches_oracle(rb, causal):
    import torch
    from burn_rocket_b200.qwen3 import Qwen3Config, Qwen3Embedding
    from oracle import qwen3_ref
    cfg = replace(Qwen3Config(), layers=2, vocab=4096)
    batch, seq = 2, 128
    hw = qwen3_ref.make_host_weights(cfg, seed=7)
    model = Qwen3Embedding(cfg, batch, seq, host_weights=hw, causal=causal)
    rng = np.random.default_rng(8)
    ids = rng.integers(0, cfg.vocab, size=batch * seq, dtype=np.int32)
    model.ids.copy_(torch.from_numpy(ids))
    got = model.forward_device().cpu().numpy()
    rb.check_device_errors()
    want = qwen3_ref.forward(hw, cfg, ids, batch, seq, causal)
    for b in range(batch):
        assert cosine(got[b], want[b]) >= 0.9999, (b, cosine(got[b], want[b]))
    assert max_rel(got, want) <= 1e-2
    # the CUDA-graph replay gives the same result
    model.capture()
    assert np.array_equal(model.run().cpu().numpy(), got)
