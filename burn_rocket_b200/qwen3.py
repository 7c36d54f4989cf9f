"""Qwen3-Embedding-architecture forward on librocket_b200 (BASELINE config #3).

Mirrors src/qwen3_embedding/model.rs: per layer
    h = rms_norm(x)                                  (model.rs:261-291)
    q|k|v = h · Wqkv^T  (one fused Q8_0 matmul)      (model.rs:355-368, pack3)
    q, k = rope(rms_norm_per_head(q)), rope(rms_norm_per_head(k))   (model.rs:369-376)
    x += attention(q, k, v) · Wo^T
    h = rms_norm(x)
    x += (silu(h · Wg^T) * (h · Wu^T)) · Wd^T        (model.rs:593-606, pack2 gate|up)
then the final rms_norm of each sequence's last token (model.rs:230-235),
L2-normalised as config #3 asks. Attention is bidirectional for config #3 and
causal in the reference model (`causal=True` gives the reference's mask).

Every op is a librocket_b200 kernel launched through the C ABI: Q8_0 tcgen05
GEMMs, the fused flash attention reading q/k/v straight from the q|k|v
buffer, and the fused glue (embedding gather, residual-add + RMSNorm, per-head
RMSNorm + RoPE, SiLU·mul, last-token norm + L2). torch only allocates device
buffers, generates the synthetic weights and captures the call sequence into
a CUDA graph. The residual stream is f32; matmul inputs/outputs are f16 (the
reference's NPU route also rounds matmul operands and outputs to f16,
ext.rs:1437-1499).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from . import _lib
from . import _check, _dev_ptr, _stream_ptr, WeightId, matmul, pack_gated_q8_0
from ._lib import DTYPE_F16, MASK_CAUSAL, MASK_NONE


@dataclass(frozen=True)
class Qwen3Config:
    layers: int = 28
    hidden: int = 1024
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 3072
    vocab: int = 151669
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def linear_params_per_layer(self) -> int:
        h, d = self.hidden, self.head_dim
        return (h * (self.heads + 2 * self.kv_heads) * d + self.heads * d * h + 3 * h * self.inter)

    def flops_per_token(self, seq: int) -> float:
        """Algorithmic FLOPs per token: linear 2·params + attention 4·S·D·H, per layer."""
        return self.layers * (2.0 * self.linear_params_per_layer + 4.0 * seq * self.head_dim * self.heads)


def rope_tables(seq: int, head_dim: int, theta: float):
    """cos/sin [seq, head_dim/2] f32: inv_freq in f64 cast to f32, angle in f32
    (src/util/rope.rs:15-31)."""
    half = head_dim // 2
    inv = np.array([1.0 / theta ** (2.0 * i / head_dim) for i in range(half)], np.float64).astype(np.float32)
    pos = np.arange(seq, dtype=np.float32)
    ang = (pos[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class Qwen3Embedding:
    """Resident random-init model (Q8_0 linears) + preallocated activations for
    `batch` sequences of `seq` tokens on the current CUDA device."""

    def __init__(self, cfg: Qwen3Config, batch: int, seq: int, seed: int = 0, causal: bool = False,
                 host_weights: dict | None = None, norm_ones: bool = True):
        import torch
        self.cfg, self.batch, self.seq, self.causal = cfg, batch, seq, causal
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        T = batch * seq
        self.T = T
        lib = _lib.load()
        g = torch.Generator(device=dev).manual_seed(seed)
        h, hd, nh, nkv, inter = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.inter
        self.layers = []

        def randn(*shape):
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * 0.02).contiguous()

        def pack_dev(parts):
            ptrs = (C.c_void_p * len(parts))(*[p.data_ptr() for p in parts])
            ns = (C.c_int64 * len(parts))(*[p.shape[0] for p in parts])
            wid = lib.rb_pack_f32_q8_0_device(ptrs, ns, len(parts), parts[0].shape[1])
            _check(wid, "rocket_pack", 0, parts[0].shape[1], sum(p.shape[0] for p in parts))
            return WeightId(int(wid))

        def norm_w(n):
            if norm_ones:
                return torch.ones(n, device=dev)
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).contiguous()

        for li in range(cfg.layers):
            if host_weights is not None:
                W = {k: torch.from_numpy(v).to(dev) for k, v in host_weights["layers"][li].items()}
            else:
                W = {"wq": randn(nh * hd, h), "wk": randn(nkv * hd, h), "wv": randn(nkv * hd, h),
                     "wo": randn(h, nh * hd), "wg": randn(inter, h), "wu": randn(inter, h), "wd": randn(h, inter),
                     "in_norm": norm_w(h), "post_norm": norm_w(h), "q_norm": norm_w(hd), "k_norm": norm_w(hd)}
            layer = {
                "qkv": pack_dev([W["wq"], W["wk"], W["wv"]]),   # pack3
                "o": pack_dev([W["wo"]]),
                "gu": pack_gated_q8_0(W["wg"], W["wu"]),       # pack2 + fused silu_mul
                "down": pack_dev([W["wd"]]),
                "in_norm": W["in_norm"].float().contiguous(), "post_norm": W["post_norm"].float().contiguous(),
                "q_norm": W["q_norm"].float().contiguous(), "k_norm": W["k_norm"].float().contiguous(),
            }
            del W
            self.layers.append(layer)
        if host_weights is not None:
            self.embed = torch.from_numpy(host_weights["embed"]).to(dev).half().contiguous()
            self.final_norm = torch.from_numpy(host_weights["final_norm"]).to(dev).float().contiguous()
        else:
            self.embed = (torch.randn(cfg.vocab, h, generator=g, device=dev) * 0.02).half().contiguous()
            self.final_norm = norm_w(h).float().contiguous()
        cos, sin = rope_tables(seq, hd, cfg.theta)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        torch.cuda.synchronize()
        # activations
        f16 = torch.float16
        self.ids = torch.zeros(T, dtype=torch.int32, device=dev)
        self.x = torch.empty(T, h, dtype=torch.float32, device=dev)
        self.h = torch.empty(T, h, dtype=f16, device=dev)
        self.qkv = torch.empty(T, (nh + 2 * nkv) * hd, dtype=f16, device=dev)
        self.attn = torch.empty(T, nh * hd, dtype=f16, device=dev)
        self.o = torch.empty(T, h, dtype=f16, device=dev)
        self.act = torch.empty(T, inter, dtype=f16, device=dev)
        self.d = torch.empty(T, h, dtype=f16, device=dev)
        self.out = torch.empty(batch, h, dtype=torch.float32, device=dev)
        self.graph = None

    # ------------------------------------------------------------------ forward
    def _layer(self, L: dict, delta, stream=None):
        """One decoder layer on the residual stream self.x: `delta` (a device
        pointer or None) is the previous layer's pending MLP output, folded into
        this layer's first residual-add + RMSNorm. Returns this layer's pending
        MLP output pointer."""
        cfg, lib, T = self.cfg, _lib.load(), self.T
        st = _stream_ptr(stream)
        h, hd, nh, nkv = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
        ld = (nh + 2 * nkv) * hd
        qkv_p = _dev_ptr(self.qkv)
        _check(lib.rb_add_rms_norm(_dev_ptr(self.x), delta, _dev_ptr(L["in_norm"]), cfg.eps, _dev_ptr(self.h),
                                   T, h, st), "add_rms_norm")
        matmul(self.h, L["qkv"], out=self.qkv, stream=stream)
        _check(lib.rb_qk_norm_rope(qkv_p, ld, T, nh, nkv, hd, _dev_ptr(L["q_norm"]), _dev_ptr(L["k_norm"]),
                                   cfg.eps, _dev_ptr(self.cos), _dev_ptr(self.sin), self.seq, st),
               "qk_norm_rope")
        _check(lib.rb_attention_batched(qkv_p, ld, qkv_p + nh * hd * 2, ld, qkv_p + (nh + nkv) * hd * 2, ld,
                                        _dev_ptr(self.attn), nh * hd, DTYPE_F16, self.batch, self.seq, self.seq,
                                        nh, nkv, hd, 1.0 / math.sqrt(hd), 0.0,
                                        MASK_CAUSAL if self.causal else MASK_NONE, -1, 0, 0, st),
               "rocket_flash_attn", self.seq, self.seq, hd)
        matmul(self.attn, L["o"], out=self.o, stream=stream)
        _check(lib.rb_add_rms_norm(_dev_ptr(self.x), _dev_ptr(self.o), _dev_ptr(L["post_norm"]), cfg.eps,
                                   _dev_ptr(self.h), T, h, st), "add_rms_norm")
        matmul(self.h, L["gu"], out=self.act, stream=stream)  # silu(h Wg^T) * (h Wu^T)
        matmul(self.act, L["down"], out=self.d, stream=stream)
        return _dev_ptr(self.d)

    def forward_device(self, stream=None):
        """One forward over self.ids (device int32 [T]) into self.out [batch, hidden]."""
        cfg, lib, T = self.cfg, _lib.load(), self.T
        st = _stream_ptr(stream)
        h = cfg.hidden
        self.embed_device(stream)
        delta = None
        for L in self.layers:
            delta = self._layer(L, delta, stream)
        # final residual, then the last token's norm + L2
        _check(lib.rb_add_rms_norm(_dev_ptr(self.x), delta, _dev_ptr(self.final_norm), cfg.eps, _dev_ptr(self.h),
                                   T, h, st), "add_rms_norm")
        _check(lib.rb_last_token_l2(_dev_ptr(self.x), self.batch, self.seq, h, _dev_ptr(self.final_norm), cfg.eps,
                                    _dev_ptr(self.out), st), "last_token_l2")
        return self.out

    def embed_device(self, stream=None):
        """self.x = the f32 embedding rows of self.ids (the residual stream's start)."""
        cfg, lib = self.cfg, _lib.load()
        _check(lib.rb_embed_gather(_dev_ptr(self.ids), self.T, _dev_ptr(self.embed), cfg.vocab, cfg.hidden,
                                   _dev_ptr(self.x), _stream_ptr(stream)), "embed_gather")
        return self.x

    def layer_step(self, li: int, stream=None):
        """Layer li alone on self.x, leaving its output residual stream in self.x
        (the pending MLP output folded in; self.h is scratch): a per-layer view
        of forward_device for checking each layer from the device's own input."""
        cfg, lib = self.cfg, _lib.load()
        delta = self._layer(self.layers[li], None, stream)
        _check(lib.rb_add_rms_norm(_dev_ptr(self.x), delta, _dev_ptr(self.final_norm), cfg.eps, _dev_ptr(self.h),
                                   self.T, cfg.hidden, _stream_ptr(stream)), "add_rms_norm")
        return self.x

    def capture(self):
        """Capture forward_device into a CUDA graph (after one eager warm-up)."""
        import torch
        self.forward_device()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self.forward_device()
        self.graph = g
        return g

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.forward_device()
        return self.out

    def embed_host(self, ids_host, out_host=None):
        """End-to-end call: host token ids [batch*seq] int32 in, host embeddings out."""
        import torch
        self.ids.copy_(ids_host, non_blocking=True)
        self.run()
        if out_host is None:
            out_host = torch.empty(self.batch, self.cfg.hidden, dtype=torch.float32, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return out_host
