"""CPU restatement of the SigLIP-style W8A8 tower (TEST INFRASTRUCTURE ONLY).

The tower is a synthetic architecture (pre-LayerNorm encoder, 16 heads x 72,
GELU-tanh MLP): its projections follow the reference's W8A8 op exactly —
per-output-channel int8 weight codes (orc_quantize_weight_per_channel, the
form pack_qat consumes, crates/burn-rocket/src/ext.rs:1382-1425) and dynamic
per-token activation codes with the int32 accumulate and f32 epilogue of
matmul_qat (ext.rs:1245-1373), via the C oracle. Attention is the bidirectional
softmax(QK^T/sqrt(72))V of attention_window(-1) (ext.rs:1907-1950), GELU the
tanh form of crates/burn-rocket/src/host.rs:15-18, LayerNorm the biased-variance
form with eps inside the square root. Activations are rounded to f16 where the
device stores them in f16 (matmul inputs and outputs); everything else is f64.
"""
from __future__ import annotations

import numpy as np

from . import oracle as orc


def make_host_weights(cfg, seed: int, affine: bool = True) -> dict:
    """Seeded synthetic weights (numpy f32; linears f16-representable) in the layout
    SiglipTower(host_weights=) takes."""
    rng = np.random.default_rng(seed)
    h, hq, inter = cfg.hidden, cfg.heads * cfg.head_dim, cfg.inter

    def randn16(*shape):
        w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        return w.astype(np.float16).astype(np.float32)

    def ln(n):
        if not affine:
            return np.ones(n, np.float32), np.zeros(n, np.float32)
        return ((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32),
                (0.05 * rng.standard_normal(n)).astype(np.float32))

    layers = []
    for _ in range(cfg.layers):
        g1, b1 = ln(h)
        g2, b2 = ln(h)
        layers.append({"wq": randn16(hq, h), "wk": randn16(hq, h), "wv": randn16(hq, h), "wo": randn16(h, hq),
                       "w1": randn16(inter, h), "w2": randn16(h, inter),
                       "ln1_g": g1, "ln1_b": b1, "ln2_g": g2, "ln2_b": b2})
    pg, pb = ln(h)
    return {"layers": layers, "post_g": pg, "post_b": pb}


def _f16(x):
    return np.asarray(x, np.float64).astype(np.float32).astype(np.float16).astype(np.float64)


def layer_norm(x, g, b, eps):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * g + b


def layer_norm_f32(x, g, b, eps):
    """The same LayerNorm evaluated in f32 (as an f32 CPU path computes it):
    the chain's sensitivity to rounding-level differences."""
    x = np.asarray(x, np.float32)
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    var = ((x - mu) ** 2).mean(-1, keepdims=True, dtype=np.float32)
    y = (x - mu) / np.sqrt(var + np.float32(eps)) * np.asarray(g, np.float32) + np.asarray(b, np.float32)
    return y.astype(np.float64)


def gelu_tanh(x):
    """host.rs:15-18: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * (x * x * x))))


def _w8a8(x16, w):
    codes, ws = orc.quantize_weight_per_channel(w)
    return orc.w8a8_matmul(np.asarray(x16, np.float32), codes, ws).astype(np.float64)


def attention(qkv, cfg, images: int, f16_inputs: bool = False) -> np.ndarray:
    """Bidirectional softmax(q k^T / sqrt(D)) v per image and head over a fused
    q|k|v [images*patches, 3*heads*D] buffer (f64). f16_inputs: the buffer
    holds f16 values, so the C oracle's flash_attn_ref (attn/oneshot.rs:130-199,
    f64 arithmetic, f16 result) computes it."""
    S, H, D = cfg.patches, cfg.heads, cfg.head_dim
    hq = H * D
    att = np.empty((images * S, hq))
    if f16_inputs:
        bits = orc.f32_to_f16_bits(np.asarray(qkv, np.float32))
        for im in range(images):
            rows = slice(im * S, (im + 1) * S)
            q, k, v = (np.ascontiguousarray(bits[rows, i * hq:(i + 1) * hq]) for i in range(3))
            att[rows] = orc.f16_bits_to_f32(orc.flash_attn_ref(q, k, v, H, H, D, 1.0 / np.sqrt(D)))
        return att
    for im in range(images):
        rows = slice(im * S, (im + 1) * S)
        for hh in range(H):
            q = qkv[rows, hh * D:(hh + 1) * D]
            k = qkv[rows, hq + hh * D:hq + (hh + 1) * D]
            v = qkv[rows, 2 * hq + hh * D:2 * hq + (hh + 1) * D]
            s = q @ k.T / np.sqrt(D)
            p = np.exp(s - s.max(-1, keepdims=True))
            att[rows, hh * D:(hh + 1) * D] = (p / p.sum(-1, keepdims=True)) @ v
    return att


def layer(L: dict, cfg, x: np.ndarray, images: int, quant: bool = True, ln32: bool = False) -> np.ndarray:
    """One pre-LN encoder layer on the f64 residual stream x [images*patches,
    hidden]; returns the new residual stream. quant=True follows the device's
    W8A8 projections and f16 activations (GELU of the f32 fc1 product, then
    the f16 store, as the fused fc1 epilogue does); quant=False is the float
    skeleton (f64 throughout, no codes). ln32: the pre-norms in f32."""
    norm = layer_norm_f32 if ln32 else layer_norm
    if quant:
        f16, lin = _f16, _w8a8
    else:
        f16 = lambda a: np.asarray(a, np.float64)  # noqa: E731
        lin = lambda a, w: np.asarray(a, np.float64) @ np.asarray(w, np.float64).T  # noqa: E731
    x = np.asarray(x, np.float64)
    wqkv = np.concatenate([L["wq"], L["wk"], L["wv"]], 0)
    h16 = f16(norm(x, L["ln1_g"], L["ln1_b"], cfg.eps))
    qkv = f16(lin(h16, wqkv))
    att = attention(qkv, cfg, images, f16_inputs=quant)
    x = x + f16(lin(f16(att), L["wo"]))
    h16 = f16(norm(x, L["ln2_g"], L["ln2_b"], cfg.eps))
    f = f16(gelu_tanh(lin(h16, L["w1"])))
    return x + f16(lin(f, L["w2"]))


def forward(hw: dict, cfg, patches: np.ndarray, images: int, quant: bool = True, ln32: bool = False) -> np.ndarray:
    """Final-LayerNorm patch states [images*patches, hidden] (f64)."""
    x = np.asarray(patches, np.float64).reshape(images * cfg.patches, cfg.hidden).copy()
    for L in hw["layers"]:
        x = layer(L, cfg, x, images, quant, ln32)
    return layer_norm(x, hw["post_g"], hw["post_b"], cfg.eps)
