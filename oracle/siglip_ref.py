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


def gelu_tanh(x):
    """host.rs:15-18: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def _w8a8(x16, w):
    codes, ws = orc.quantize_weight_per_channel(w)
    return orc.w8a8_matmul(np.asarray(x16, np.float32), codes, ws).astype(np.float64)


def forward(hw: dict, cfg, patches: np.ndarray, images: int) -> np.ndarray:
    """Final-LayerNorm patch states [images*patches, hidden] (f64)."""
    S, H, D = cfg.patches, cfg.heads, cfg.head_dim
    hq = H * D
    x = np.asarray(patches, np.float64).reshape(images * S, cfg.hidden).copy()
    for L in hw["layers"]:
        wqkv = np.concatenate([L["wq"], L["wk"], L["wv"]], 0)
        h16 = _f16(layer_norm(x, L["ln1_g"], L["ln1_b"], cfg.eps))
        qkv = _f16(_w8a8(h16, wqkv))
        att = np.empty((images * S, hq))
        for im in range(images):
            rows = slice(im * S, (im + 1) * S)
            for hh in range(H):
                q = qkv[rows, hh * D:(hh + 1) * D]
                k = qkv[rows, hq + hh * D:hq + (hh + 1) * D]
                v = qkv[rows, 2 * hq + hh * D:2 * hq + (hh + 1) * D]
                s = q @ k.T / np.sqrt(D)
                p = np.exp(s - s.max(-1, keepdims=True))
                att[rows, hh * D:(hh + 1) * D] = (p / p.sum(-1, keepdims=True)) @ v
        x = x + _f16(_w8a8(_f16(att), L["wo"]))
        h16 = _f16(layer_norm(x, L["ln2_g"], L["ln2_b"], cfg.eps))
        f16 = _f16(gelu_tanh(_f16(_w8a8(h16, L["w1"]))))
        x = x + _f16(_w8a8(f16, L["w2"]))
    return layer_norm(x, hw["post_g"], hw["post_b"], cfg.eps)
