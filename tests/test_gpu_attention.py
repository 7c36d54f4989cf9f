"""Device parity of the fused GQA flash-attention kernel, through the C ABI.

Small and ragged cases compare against the CPU oracle (flash_attn_ref of
attn/oneshot.rs:130-185 with the masks.rs predicates); the full BASELINE
config #2 size compares against the oracle on one KV group and against a plain
torch fp32 reference of the same op on all heads.
Tolerance (north star): cosine >= 0.9999 and max |err| <= 1e-2 * max |ref|.
"""
import math

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
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / (np.abs(want).max() + 1e-30))


def run_case(rb, orc, n_q, n_kv, h, hkv, d, mode, window=-1, q0=0, k0=0, softcap=0.0, seed=0,
             dtype="f16"):
    import torch
    rng = np.random.default_rng(seed)
    q = orc.f32_to_f16_bits(rng.standard_normal((n_q, h * d)).astype(np.float32))
    k = orc.f32_to_f16_bits(rng.standard_normal((n_kv, hkv * d)).astype(np.float32))
    v = orc.f32_to_f16_bits(rng.standard_normal((n_kv, hkv * d)).astype(np.float32))
    scale = 1.0 / math.sqrt(d)
    ref = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, h, hkv, d, scale, softcap, mode, window, q0, k0))
    tq, tk, tv = (torch.from_numpy(a.view(np.float16)).cuda() for a in (q, k, v))
    if dtype == "f32":
        tq, tk, tv = tq.float(), tk.float(), tv.float()
    out = rb.attention_raw(tq, tk, tv, h, hkv, d, scale, softcap, mode, window, q0, k0)
    torch.cuda.synchronize()
    rb.check_device_errors()
    return out.float().cpu().numpy(), ref


M = None  # filled lazily from the oracle module


CASES = [
    # n_q, n_kv, h, hkv, d, mode, window, q0, k0
    (1, 1, 2, 1, 128, 0, -1, 0, 0),
    (77, 77, 2, 1, 128, 0, -1, 0, 0),
    (128, 128, 4, 2, 128, 2, -1, 0, 0),
    (300, 300, 16, 8, 128, 2, -1, 0, 0),
    (300, 300, 16, 8, 128, 0, -1, 0, 0),
    (257, 257, 8, 8, 64, 2, -1, 0, 0),
    (200, 200, 32, 4, 128, 2, -1, 0, 0),
    (333, 333, 4, 2, 64, 3, 37, 0, 0),
    (333, 333, 4, 2, 128, 4, 50, 0, 0),
    (150, 400, 4, 2, 128, 5, 60, 200, 150),
    (150, 500, 4, 2, 128, 6, -1, 300, 0),
    (150, 400, 4, 2, 64, 6, 90, 300, 100),
    (64, 300, 2, 1, 128, 1, -1, 0, 0),
    # one or two long units: each is cut over many CTAs and merged by the last part
    (64, 4096, 2, 1, 128, 1, -1, 0, 0),
    (200, 6000, 2, 2, 128, 1, -1, 0, 0),
    (256, 9000, 2, 1, 64, 6, -1, 8744, 0),
    # bands that start or end one key either side of a 128-key tile edge
    (256, 256, 4, 2, 128, 4, 127, 0, 0),
    (256, 384, 4, 2, 128, 5, 128, 129, 1),
    (129, 257, 2, 1, 128, 6, 129, 128, 0),
    (257, 257, 2, 2, 64, 3, 129, 0, 0),
    # head_dim 72 (staged as 80 = 64-column atom + 16-column tail)
    (1, 1, 2, 2, 72, 0, -1, 0, 0),
    (300, 300, 16, 16, 72, 0, -1, 0, 0),
    (257, 257, 4, 2, 72, 2, -1, 0, 0),
    (150, 400, 4, 2, 72, 5, 60, 200, 150),
    (255, 255, 2, 2, 72, 3, 128, 0, 0),
]


@pytest.fixture(params=["never", "always"])
def split(rb, request):
    """Both work schedules: one CTA per query-slot pair and KV head, and one
    CTA per SM over equal key-tile shares with split units merged."""
    old = rb.set_attention_split(request.param)
    yield request.param
    rb.set_attention_split(old)


@pytest.mark.parametrize("case", CASES)
def test_attention_matches_oracle(rb, orc, case, split):
    n_q, n_kv, h, hkv, d, mode, window, q0, k0 = case
    got, ref = run_case(rb, orc, n_q, n_kv, h, hkv, d, mode, window, q0, k0, seed=sum(case[:5]))
    assert cosine(got, ref) >= COS_MIN, cosine(got, ref)
    assert max_rel(got, ref) <= MAX_REL, max_rel(got, ref)


def test_attention_split_policy_contract(rb):
    import burn_rocket_b200._lib as L
    assert L.load().rb_set_attention_split(7) != 0
    with pytest.raises(ValueError):
        rb.set_attention_split("sometimes")


def test_attention_split_units_deterministic(rb, orc, split):
    """Units cut over CTAs merge in CTA order whichever part arrives last, and
    the arrival counters reset themselves: repeated calls agree bit for bit."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(3)
    n_q, n_kv, h, hkv, d = 200, 7000, 4, 2, 128
    q = torch.randn(n_q, h * d, device="cuda", generator=g).half()
    k = torch.randn(n_kv, hkv * d, device="cuda", generator=g).half()
    v = torch.randn(n_kv, hkv * d, device="cuda", generator=g).half()
    outs = [rb.attention_raw(q, k, v, h, hkv, d, 1.0 / math.sqrt(d), 0.0, 1, -1, 0, 0).clone() for _ in range(4)]
    torch.cuda.synchronize()
    rb.check_device_errors()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_attention_softcap(rb, orc):
    got, ref = run_case(rb, orc, 200, 200, 4, 2, 128, 2, softcap=5.0, seed=3)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL


def test_attention_fully_masked_rows_average_every_key(rb, orc):
    """A causal block whose keys lie above some queries: those rows see no key
    and average every real key (attn/oneshot.rs:910-950)."""
    got, ref = run_case(rb, orc, 130, 200, 2, 1, 128, 6, -1, q0=0, k0=60, seed=4)
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL


def test_attention_f32_boundary(rb, orc):
    got, ref = run_case(rb, orc, 160, 160, 4, 2, 128, 2, seed=5, dtype="f32")
    assert cosine(got, ref) >= COS_MIN
    assert max_rel(got, ref) <= MAX_REL


def torch_ref(q, k, v, h, hkv, d, causal):
    import torch
    n = q.shape[0]
    g = h // hkv
    qf = q.float().view(n, h, d).transpose(0, 1)
    kf = k.float().view(-1, hkv, d).transpose(0, 1).repeat_interleave(g, 0)
    vf = v.float().view(-1, hkv, d).transpose(0, 1).repeat_interleave(g, 0)
    s = (qf @ kf.transpose(1, 2)) / math.sqrt(d)
    if causal:
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(0, 1).reshape(n, h * d)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_attention_config2_full_size(rb, causal, dtype, split):
    """BASELINE config #2: 3633 tokens, 16/8 heads x 128, causal and bidirectional."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(7)
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    n, h, hkv, d = 3633, 16, 8, 128
    q = torch.randn(n, h * d, device="cuda", generator=g).to(tdt)
    k = torch.randn(n, hkv * d, device="cuda", generator=g).to(tdt)
    v = torch.randn(n, hkv * d, device="cuda", generator=g).to(tdt)
    out = rb.attention(q, k, v, h, hkv, d, 1.0 / math.sqrt(d), None, causal)
    torch.cuda.synchronize()
    rb.check_device_errors()
    ref = torch_ref(q, k, v, h, hkv, d, causal)
    got = out.float()
    cos = torch.nn.functional.cosine_similarity(got.flatten().double(), ref.flatten().double(), dim=0).item()
    mr = ((got - ref).abs().max() / ref.abs().max()).item()
    assert cos >= COS_MIN, cos
    assert mr <= MAX_REL, mr


@pytest.mark.parametrize("causal", [True, False])
def test_attention_config2_full_size_vs_oracle(rb, orc, causal):
    """BASELINE config #2 at full size (3633 tokens, 16/8 heads x 128, RoPE
    theta 1e6 pre-applied, fp16) against the oracle's flash_attn_ref
    (attn/oneshot.rs:130-199, f64, the -30000 clamp) on one KV group: query
    heads 10 and 11, which read KV head 5."""
    import torch
    n, h, hkv, d = 3633, 16, 8, 128
    rng = np.random.default_rng(36)
    half = d // 2
    inv = np.array([1.0 / 1e6 ** (2.0 * i / d) for i in range(half)], np.float64).astype(np.float32)
    ang = (np.arange(n, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]

    def roped(heads):
        x = rng.standard_normal((n, heads, d)).astype(np.float32)
        x1, x2 = x[..., :half], x[..., half:]
        return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).reshape(n, heads * d)

    q = orc.f32_to_f16_bits(roped(h))
    k = orc.f32_to_f16_bits(roped(hkv))
    v = orc.f32_to_f16_bits(rng.standard_normal((n, hkv * d)).astype(np.float32))
    tq, tk, tv = (torch.from_numpy(a.view(np.float16)).cuda() for a in (q, k, v))
    out = rb.attention(tq, tk, tv, h, hkv, d, 1.0 / math.sqrt(d), None, causal)
    torch.cuda.synchronize()
    rb.check_device_errors()
    got = out.float().cpu().numpy()[:, 10 * d:12 * d]
    mode = orc.MASK_CAUSAL if causal else orc.MASK_NONE
    ref = orc.f16_bits_to_f32(orc.flash_attn_ref(np.ascontiguousarray(q[:, 10 * d:12 * d]),
                                                 np.ascontiguousarray(k[:, 5 * d:6 * d]),
                                                 np.ascontiguousarray(v[:, 5 * d:6 * d]), 2, 1, d,
                                                 1.0 / math.sqrt(d), 0.0, mode))
    assert cosine(got, ref) >= COS_MIN, cosine(got, ref)
    assert max_rel(got, ref) <= MAX_REL, max_rel(got, ref)


def test_attention_host_entry(rb, orc):
    import burn_rocket_b200._lib as L
    rng = np.random.default_rng(8)
    n, h, hkv, d = 100, 4, 2, 128
    q = orc.f32_to_f16_bits(rng.standard_normal((n, h * d)).astype(np.float32))
    k = orc.f32_to_f16_bits(rng.standard_normal((n, hkv * d)).astype(np.float32))
    v = orc.f32_to_f16_bits(rng.standard_normal((n, hkv * d)).astype(np.float32))
    out = np.empty_like(q)
    rc = L.load().rb_attention_host(q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data, L.DTYPE_F16,
                                    n, n, h, hkv, d, 1.0 / math.sqrt(d), 0.0, L.MASK_CAUSAL, -1, 0, 0)
    assert rc == 0, L.last_error()
    ref = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, h, hkv, d, 1.0 / math.sqrt(d), 0.0, 2))
    got = orc.f16_bits_to_f32(out)
    assert cosine(got, ref) >= COS_MIN and max_rel(got, ref) <= MAX_REL


@pytest.mark.parametrize("mode,window,dim", [("causal", -1, 128), ("none", -1, 128), ("window", 300, 64),
                                             ("causal_window", 500, 128), ("causal", -1, 72)])
def test_attention_host_entry_pipelined(rb, mode, window, dim):
    """Long full-sequence calls of rb_attention_host run in overlapped
    query-row chunks (copy in, attention, copy out); the result equals the
    device entry on the same inputs (up to f32 summation order), from pinned
    and from pageable host buffers."""
    import torch
    import burn_rocket_b200._lib as L
    modes = {"none": L.MASK_NONE, "causal": L.MASK_CAUSAL, "window": L.MASK_WINDOW,
             "causal_window": L.MASK_CAUSAL_WINDOW}
    n, h, hkv = 2500, 4, 2
    g = torch.Generator().manual_seed(n + dim + window)
    q = torch.randn(n, h * dim, generator=g).half()
    k = torch.randn(n, hkv * dim, generator=g).half()
    v = torch.randn(n, hkv * dim, generator=g).half()
    scale = 1.0 / math.sqrt(dim)
    ref = rb.attention_raw(q.cuda(), k.cuda(), v.cuda(), h, hkv, dim, scale, None, modes[mode], window)
    torch.cuda.synchronize()
    ref = ref.float().cpu()
    for pinned in (True, False):
        qh, kh, vh = (t.pin_memory() if pinned else t.clone() for t in (q, k, v))
        out = torch.empty_like(qh).pin_memory() if pinned else torch.empty_like(qh)
        rc = L.load().rb_attention_host(qh.data_ptr(), kh.data_ptr(), vh.data_ptr(), out.data_ptr(), L.DTYPE_F16,
                                        n, n, h, hkv, dim, scale, 0.0, modes[mode], window, 0, 0)
        assert rc == 0, L.last_error()
        got = out.float()
        cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
        mr = ((got - ref).abs().max() / ref.abs().max()).item()
        assert cos >= COS_MIN, cos
        assert mr <= MAX_REL, mr
    rb.check_device_errors()


def test_attention_contract_errors(rb):
    import torch
    q = torch.zeros(8, 4 * 96, dtype=torch.float16, device="cuda")
    with pytest.raises(rb.OpFailure) as ei:
        rb.attention(q, q[:, :2 * 96].contiguous(), q[:, :2 * 96].contiguous(), 4, 2, 96, 0.1)
    assert ei.value.error.rc == -5  # head_dim not supported by this build
    q = torch.zeros(8, 3 * 128, dtype=torch.float16, device="cuda")
    kv = torch.zeros(8, 2 * 128, dtype=torch.float16, device="cuda")
    with pytest.raises(rb.OpFailure) as ei:
        rb.attention(q, kv, kv, 3, 2, 128, 0.1)
    assert ei.value.error.rc == -1  # n_head % n_kv_heads
    q = torch.zeros(8, 2 * 128, dtype=torch.float16, device="cuda")
    kv = torch.zeros(9, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(rb.OpFailure) as ei:
        rb.attention(q, kv, kv, 2, 1, 128, 0.1, None, True)
    assert ei.value.error.rc == -1  # full-sequence modes need n_q == n_kv


# ------------------------------------------------------------------ chunked causal helper (a12)
@pytest.mark.parametrize("window", [None, 300])
def test_chunked_causal_attention_matches_dense(rb, orc, window):
    """causal_attention (src/util/causal.rs:103-163) with 512-row chunks equals
    the dense causal(-window) op within tolerance (the chunked calls tile and
    split the key range differently, so the f32 sums round differently)."""
    import torch
    from burn_rocket_b200.causal import causal_attention
    S, H, KV, D = 1500, 8, 2, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(S, H * D, device="cuda", generator=g).half()
    k = torch.randn(S, KV * D, device="cuda", generator=g).half()
    v = torch.randn(S, KV * D, device="cuda", generator=g).half()
    scale = 1 / math.sqrt(D)
    dense = causal_attention(q, k, v, H, KV, D, scale, window=window, chunk=0)
    chunked = causal_attention(q, k, v, H, KV, D, scale, window=window, chunk=512)
    torch.cuda.synchronize()
    a, b = dense.float().cpu().numpy(), chunked.float().cpu().numpy()
    assert cosine(a, b) >= 0.99999
    assert max_rel(b, a) <= 2e-3
    rb.check_device_errors()
