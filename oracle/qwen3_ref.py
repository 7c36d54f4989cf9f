"""CPU restatement of the Qwen3-Embedding forward (TEST INFRASTRUCTURE ONLY).

Follows src/qwen3_embedding/model.rs (layer 261-291, attention projection and
per-head q/k RMSNorm + RoPE 345-381, MLP 593-606, final norm + last token
207-236) with RoPE tables of src/util/rope.rs:15-75 and the RMSNorm / SiLU
formulas of crates/burn-rocket/src/host.rs:31-56. Linear weights are the
Q8_0-dequantised values (oracle.q8_0_quantize / q8_0_dequant, the reference's
encoder and GGUF decode); the embedding table is the f16 rounding of the f32
table (the reference keeps it in a 16-bit dtype, model.rs:218-222). Arithmetic
in f64 — the reference f32 path the device result is compared against.
"""
from __future__ import annotations

import numpy as np

from . import oracle as orc


def make_host_weights(cfg, seed: int, norm_ones: bool = False) -> dict:
    """Seeded synthetic weights (numpy f32) in the layout Qwen3Embedding(host_weights=) takes."""
    rng = np.random.default_rng(seed)
    h, hd, nh, nkv, inter = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.inter

    def randn(*shape):
        return (rng.standard_normal(shape) * 0.02).astype(np.float32)

    def norm_w(n):
        return np.ones(n, np.float32) if norm_ones else (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for _ in range(cfg.layers):
        layers.append({"wq": randn(nh * hd, h), "wk": randn(nkv * hd, h), "wv": randn(nkv * hd, h),
                       "wo": randn(h, nh * hd), "wg": randn(inter, h), "wu": randn(inter, h),
                       "wd": randn(h, inter), "in_norm": norm_w(h), "post_norm": norm_w(h),
                       "q_norm": norm_w(hd), "k_norm": norm_w(hd)})
    return {"layers": layers, "embed": randn(cfg.vocab, h), "final_norm": norm_w(h)}


def _deq(w):
    codes, scales = orc.q8_0_quantize(w)
    return orc.q8_0_dequant(codes, scales).astype(np.float64)


def _rms(x, w, eps):
    ms = (x * x).mean(-1, keepdims=True)
    return x / np.sqrt(ms + eps) * w


def _rope(x, cos, sin):
    # x [..., S, H, D]; cos/sin [S, D/2]
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = cos[:, None, :]
    s = sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def rope_tables(seq: int, head_dim: int, theta: float):
    """RopeCache::new (src/util/rope.rs:15-31): inv_freq in f64 cast to f32,
    angle = pos * inv_freq in f32, cos/sin of the f32 angle."""
    half = head_dim // 2
    inv = np.array([1.0 / theta ** (2.0 * i / head_dim) for i in range(half)], np.float64).astype(np.float32)
    ang = (np.arange(seq, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def layer(L: dict, cfg, x: np.ndarray, batch: int, seq: int, causal: bool = False, quant: bool = True):
    """One decoder layer (model.rs:261-291) on the f64 residual stream x
    [batch*seq, hidden]; returns the new residual stream. quant=False uses the
    f32 weights as they are (the float skeleton, without the Q8_0 codec)."""
    h, hd, nh, nkv = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
    g = nh // nkv
    deq = _deq if quant else (lambda w: np.asarray(w, np.float64))
    x = np.asarray(x, np.float64).reshape(batch, seq, h)
    cos, sin = rope_tables(seq, hd, cfg.theta)
    cos, sin = cos.astype(np.float64), sin.astype(np.float64)
    wq, wk, wv, wo = deq(L["wq"]), deq(L["wk"]), deq(L["wv"]), deq(L["wo"])
    wg, wu, wd = deq(L["wg"]), deq(L["wu"]), deq(L["wd"])
    hh = _rms(x, L["in_norm"].astype(np.float64), cfg.eps)
    q = (hh @ wq.T).reshape(batch, seq, nh, hd)
    k = (hh @ wk.T).reshape(batch, seq, nkv, hd)
    v = (hh @ wv.T).reshape(batch, seq, nkv, hd)
    q = _rope(_rms(q, L["q_norm"].astype(np.float64), cfg.eps), cos, sin)
    k = _rope(_rms(k, L["k_norm"].astype(np.float64), cfg.eps), cos, sin)
    att = np.empty((batch, seq, nh, hd))
    for b in range(batch):
        for hh_i in range(nh):
            s = q[b, :, hh_i] @ k[b, :, hh_i // g].T / np.sqrt(hd)
            if causal:
                s = np.where(np.tril(np.ones((seq, seq), bool)), s, -np.inf)
            p = np.exp(s - s.max(-1, keepdims=True))
            att[b, :, hh_i] = (p / p.sum(-1, keepdims=True)) @ v[b, :, hh_i // g]
    x = x + att.reshape(batch, seq, nh * hd) @ wo.T
    hh = _rms(x, L["post_norm"].astype(np.float64), cfg.eps)
    gate, up = hh @ wg.T, hh @ wu.T
    x = x + (gate / (1.0 + np.exp(-gate)) * up) @ wd.T
    return x.reshape(batch * seq, h)


def embed(hw: dict, ids: np.ndarray, quant: bool = True) -> np.ndarray:
    """Embedding rows of the token ids (f16-rounded table when quant), f64 [T, hidden]."""
    emb = orc.f16_bits_to_f32(orc.f32_to_f16_bits(hw["embed"])) if quant else hw["embed"]
    return emb[np.asarray(ids).reshape(-1)].astype(np.float64)


def head(hw: dict, cfg, x: np.ndarray, batch: int, seq: int) -> np.ndarray:
    """Final RMSNorm of each sequence's last token (model.rs:230-235), L2-normalised."""
    last = _rms(np.asarray(x, np.float64).reshape(batch, seq, -1)[:, -1, :],
                hw["final_norm"].astype(np.float64), cfg.eps)
    return last / np.maximum(np.linalg.norm(last, axis=-1, keepdims=True), 1e-12)


def forward(hw: dict, cfg, ids: np.ndarray, batch: int, seq: int, causal: bool = False,
            quant: bool = True) -> np.ndarray:
    """Embeddings [batch, hidden] (L2-normalised last-token states)."""
    x = embed(hw, ids, quant)
    for L in hw["layers"]:
        x = layer(L, cfg, x, batch, seq, causal, quant)
    return head(hw, cfg, x, batch, seq)
