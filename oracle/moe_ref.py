"""CPU restatement of the Clef / Qwen3-30B-A3B-style MoE decoder layer (TEST
INFRASTRUCTURE ONLY).

Follows the reference's layer (`src/clef/model.rs:506-613`, restated from the
torch spec `tools/clef_reference.py:179-246`):

    n  = rms_norm(x) * w_in
    q  = rope(rms_norm_head(n Wq^T) * w_qn);  k = rope(rms_norm_head(n Wk^T) * w_kn);  v = n Wv^T
    h  = x + causal_gqa_attention(q, k, v) Wo^T           (positions restart per sequence)
    n2 = rms_norm(h) * w_post
    p  = softmax(n2 Wr^T);  (ids, w) = top_k(p) with ties to the lower id, w /= sum(w)
                                                          (`route`, src/clef/model.rs:462-489)
    y  = h + sum over the token's experts in ascending expert id of
             w * down_e(silu(gate_e(n2)) * up_e(n2))      (`combine`, src/clef/engine.rs:317-340)

Arithmetic is f64. `route` also returns the reference's margins
p[k-th] - p[(k+1)-th] (the near-tie gap that decides whether a selection is
stable under rounding).
"""
from __future__ import annotations

import numpy as np


def val(n: int, salt: float, scale: float) -> np.ndarray:
    """The reference tests' closed-form weights: sin(0.37 i + salt) * scale
    (src/clef/model/tests.rs:14-18), rounded to f32."""
    i = np.arange(n, dtype=np.float64)
    return (np.sin(i * 0.37 + salt) * scale).astype(np.float32)


def mini_layer_weights(cfg: dict, layer: int) -> dict:
    """Weights of the reference's mini decoder (src/clef/model/tests.rs:40-60)."""
    h, d, i, e = cfg["hidden"], cfg["head_dim"], cfg["inter"], cfg["experts"]
    s = 10.0 * layer
    return {
        "in_norm": 1.0 + val(h, s + 1, 0.1), "post_norm": 1.0 + val(h, s + 2, 0.1),
        "wq": val(cfg["heads"] * d * h, s + 3, 0.3).reshape(cfg["heads"] * d, h),
        "wk": val(cfg["kv_heads"] * d * h, s + 4, 0.3).reshape(cfg["kv_heads"] * d, h),
        "wv": val(cfg["kv_heads"] * d * h, s + 5, 0.3).reshape(cfg["kv_heads"] * d, h),
        "wo": val(h * cfg["heads"] * d, s + 6, 0.3).reshape(h, cfg["heads"] * d),
        "q_norm": 1.0 + val(d, s + 7, 0.1), "k_norm": 1.0 + val(d, s + 8, 0.1),
        "router": val(e * h, s + 9, 0.5).reshape(e, h),
        "experts": [(val(i * h, s + 20 + x, 0.3).reshape(i, h), val(i * h, s + 30 + x, 0.3).reshape(i, h),
                     val(h * i, s + 40 + x, 0.3).reshape(h, i)) for x in range(e)],
    }


def rms(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * np.asarray(w, np.float64)


def rope_tables(seq: int, head_dim: int, theta: float):
    """inv_freq = theta^(-2j/D) in f32, angle = t * inv_freq in f32 (tools/clef_reference.py:207-212)."""
    half = head_dim // 2
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim))))
    ang = (np.arange(seq, dtype=np.float32)[:, None] * inv.astype(np.float32)[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float64), np.sin(ang).astype(np.float64)


def rope(x, cos, sin):
    """Rotate-half RoPE on [S, H, D] with cos/sin [S, D/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def route(logits, top_k: int, norm: bool = True):
    """softmax -> top-k (descending, ties to the lower id) -> renormalise
    (src/clef/model.rs:462-489). Returns ids [T, k], weights [T, k], margins [T]."""
    logits = np.asarray(logits, np.float64)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    t, e = p.shape
    ids = np.empty((t, top_k), np.int64)
    w = np.empty((t, top_k), np.float64)
    margins = np.empty(t, np.float64)
    for r in range(t):
        order = sorted(range(e), key=lambda j: (-p[r, j], j))
        sel = order[:top_k]
        ids[r] = sel
        s = p[r, sel].sum()
        w[r] = p[r, sel] / s if norm else p[r, sel]
        margins[r] = p[r, order[top_k - 1]] - p[r, order[top_k]] if top_k < e else 1.0
    return ids, w, margins


def attention_causal(q, k, v, nh, nkv):
    """q [S, nh, D], k/v [S, nkv, D] -> [S, nh*D]; head h reads kv head h // (nh/nkv)."""
    s, _, d = q.shape
    g = nh // nkv
    out = np.empty((s, nh, d))
    mask = np.triu(np.ones((s, s), bool), 1)
    for hh in range(nh):
        sc = q[:, hh] @ k[:, hh // g].T / np.sqrt(d)
        sc[mask] = -np.inf
        pr = np.exp(sc - sc.max(-1, keepdims=True))
        out[:, hh] = (pr / pr.sum(-1, keepdims=True)) @ v[:, hh // g]
    return out.reshape(s, nh * d)


def experts_combine(h, n2, ids, w, experts):
    """y = h + sum over each token's experts in ascending id of w * down(silu(gate n2) * up n2)."""
    y = np.asarray(h, np.float64).copy()
    t, k = ids.shape
    for e in range(len(experts)):
        tok, slot = np.nonzero(ids == e)
        if tok.size == 0:
            continue
        gate, up, down = (np.asarray(m, np.float64) for m in experts[e])
        x = n2[tok]
        g, u = x @ gate.T, x @ up.T
        out = ((g / (1.0 + np.exp(-g))) * u) @ down.T
        y[tok] += out * w[tok, slot][:, None]
    return y


def layer_forward(x, wts: dict, cfg: dict, lens=None, force_ids=None):
    """One decoder layer over rows x [T, hidden] (records of `lens` rows, positions
    restarting per record). Returns (y, ids, weights, margins): ids and margins
    are this layer's own top-k selection, weights those the combine used.
    force_ids [T, k] replaces the selection in the combine (e.g. by the
    device's, to compare a layer across a near-tie): the weights are then this
    layer's probabilities of those experts, renormalised over them."""
    nh, nkv, d, eps = cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"]
    x = np.asarray(x, np.float64)
    t = x.shape[0]
    lens = lens or [t]
    hid = np.empty_like(x)
    off = 0
    for sr in lens:
        xr = x[off:off + sr]
        n = rms(xr, wts["in_norm"], eps)
        q = (n @ np.asarray(wts["wq"], np.float64).T).reshape(sr, nh, d)
        k = (n @ np.asarray(wts["wk"], np.float64).T).reshape(sr, nkv, d)
        v = (n @ np.asarray(wts["wv"], np.float64).T).reshape(sr, nkv, d)
        cos, sin = rope_tables(sr, d, cfg["theta"])
        q = rope(rms(q, wts["q_norm"], eps), cos, sin)
        k = rope(rms(k, wts["k_norm"], eps), cos, sin)
        ctx = attention_causal(q, k, v, nh, nkv)
        hid[off:off + sr] = xr + ctx @ np.asarray(wts["wo"], np.float64).T
        off += sr
    n2 = rms(hid, wts["post_norm"], eps)
    logits = n2 @ np.asarray(wts["router"], np.float64).T
    ids, w, margins = route(logits, cfg["top_k"], cfg.get("norm_topk", True))
    use = ids
    if force_ids is not None:
        use = np.asarray(force_ids, np.int64)
        p = np.exp(logits - logits.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        w = np.take_along_axis(p, use, 1)
        if cfg.get("norm_topk", True):
            w = w / w.sum(-1, keepdims=True)
    y = experts_combine(hid, n2, use, w, wts["experts"])
    return y, ids, w, margins


# ---------------------------------------------------------------- the device model's reference
def make_host_weights(cfg, seed: int) -> dict:
    """Seeded synthetic weights (numpy f32) in the layout MoeModel(host_weights=) takes:
    linears ~ N(0, 0.02), norm weights 1 + N(0, 0.1), embedding ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    h, d, nh, nkv, e, i = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.inter

    def randn(*shape):
        return (rng.standard_normal(shape) * 0.02).astype(np.float32)

    def norm_w(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for _ in range(cfg.layers):
        layers.append({"wq": randn(nh * d, h), "wk": randn(nkv * d, h), "wv": randn(nkv * d, h),
                       "wo": randn(h, nh * d), "router": randn(e, h),
                       "experts": [(randn(i, h), randn(i, h), randn(h, i)) for _ in range(e)],
                       "in_norm": norm_w(h), "post_norm": norm_w(h), "q_norm": norm_w(d), "k_norm": norm_w(d)})
    return {"layers": layers, "embed": randn(cfg.vocab, h), "final_norm": norm_w(h)}


class _LazyExperts:
    """experts[e] -> (gate, up, down) f64, dequantised when used (a
    full-width layer holds 128 x 3 expert matrices: too many to keep in f64)."""

    def __init__(self, experts, deq):
        self.experts, self.deq = experts, deq

    def __len__(self):
        return len(self.experts)

    def __getitem__(self, e):
        return tuple(self.deq(m) for m in self.experts[e])


def dequantised_layer(L: dict, quant: bool = True) -> dict:
    """A layer's weights as the device holds them: every linear through the
    Q8_0 codec (oracle.q8_0_quantize / q8_0_dequant) when quant, f64."""
    from . import oracle as orc

    def deq(w):
        if not quant:
            return np.asarray(w, np.float64)
        codes, scales = orc.q8_0_quantize(np.asarray(w, np.float32))
        return orc.q8_0_dequant(codes, scales).astype(np.float64)

    return {"in_norm": L["in_norm"], "post_norm": L["post_norm"], "q_norm": L["q_norm"], "k_norm": L["k_norm"],
            "wq": deq(L["wq"]), "wk": deq(L["wk"]), "wv": deq(L["wv"]), "wo": deq(L["wo"]),
            "router": deq(L["router"]), "experts": _LazyExperts(L["experts"], deq)}


def layer_cfg(cfg) -> dict:
    return {"heads": cfg.heads, "kv_heads": cfg.kv_heads, "head_dim": cfg.head_dim, "eps": cfg.eps,
            "theta": cfg.theta, "top_k": cfg.top_k, "norm_topk": True}


def forward(hw: dict, cfg, ids: np.ndarray, batch: int, seq: int, force_routing=None):
    """Final-normed hidden states [batch*seq, hidden] (f64) and per-layer
    (ids, weights, margins), with every linear weight taken through the Q8_0
    codec (oracle.q8_0_quantize / q8_0_dequant) and the embedding rounded to
    f16, as the device model stores them. force_routing: per layer, expert ids
    [T, k] that replace this chain's own selection (layer_forward force_ids)."""
    from . import oracle as orc
    c = layer_cfg(cfg)
    emb = orc.f16_bits_to_f32(orc.f32_to_f16_bits(hw["embed"]))
    x = emb[np.asarray(ids).reshape(-1)].astype(np.float64)
    routing = []
    for li, L in enumerate(hw["layers"]):
        force = None if force_routing is None else force_routing[li]
        x, rid, rw, mg = layer_forward(x, dequantised_layer(L), c, lens=[seq] * batch, force_ids=force)
        routing.append((rid, rw, mg))
    return rms(x, hw["final_norm"], cfg.eps), routing
