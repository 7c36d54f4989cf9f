"""Qwen3-30B-A3B-style MoE decoder on librocket_b200 (BASELINE config #5).

Mirrors the reference's Clef thinker layer (`src/clef/model.rs:506-613`,
torch spec `tools/clef_reference.py:179-246`): per layer

    n  = rms_norm(x)
    q|k|v = n · Wqkv^T (one fused Q8_0 matmul);  q, k = rope(rms_norm_head(q)), rope(rms_norm_head(k))
    x += causal_gqa_attention(q, k, v) · Wo^T         (positions restart per sequence)
    n2 = rms_norm(x)
    logits = n2 · Wr^T (f32);  (ids, w) = top_k(softmax(logits)), w renormalised   (model.rs:462-489)
    x += sum over each token's experts in ascending id of
         w · down_e(silu(gate_e · n2) * (up_e · n2))                               (engine.rs:284-340)

then the final RMSNorm of every token. The experts run as grouped Q8_0 GEMMs
over expert-contiguous, 256-row-aligned segments of a permuted activation
buffer (`rb_moe_dispatch`, `rb_matmul_grouped`, `rb_moe_combine`): the
experts' gate and up weights form one gated Q8_0 weight whose grouped matmul
writes silu(gate·x)·(up·x) directly (`pack_gated_q8_0`; the unfused gate|up
matmul + silu_mul when inter is not a multiple of 64), and their down blocks
another ([E * hidden, inter]). Routing,
dispatch and combine run on the device, so the whole forward is captured in
one CUDA graph. The residual stream is f32; matmul operands are f16.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from . import _lib
from . import _check, _dev_ptr, _stream_ptr, WeightId, matmul, pack_gated_q8_0
from ._lib import DTYPE_F16, DTYPE_F32, MASK_CAUSAL
from .qwen3 import rope_tables


@dataclass(frozen=True)
class MoeConfig:
    layers: int = 48
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    inter: int = 768
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 1e6

    def flops_per_token(self, seq: int) -> float:
        """Active linear 2·params (attention projections, router, top_k experts)
        plus causal attention 2·S·D·H (half of 4·S·D·H), per layer."""
        h, d = self.hidden, self.head_dim
        dense = h * (self.heads + 2 * self.kv_heads) * d + self.heads * d * h + h * self.experts
        expert = 3 * h * self.inter * self.top_k
        return self.layers * (2.0 * (dense + expert) + 2.0 * seq * d * self.heads)


class MoeModel:
    """Resident random-init model (Q8_0 linears) + preallocated activations
    for `batch` sequences of `seq` tokens on the current CUDA device."""

    def __init__(self, cfg: MoeConfig, batch: int, seq: int, seed: int = 0, host_weights: dict | None = None):
        import torch
        self.cfg, self.batch, self.seq = cfg, batch, seq
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        T = batch * seq
        self.T = T
        lib = _lib.load()
        g = torch.Generator(device=dev).manual_seed(seed)
        h, d, nh, nkv, E, I = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.inter

        def randn(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).mul_(0.02)

        def pack_dev(parts):
            parts = [p.float().contiguous() for p in parts]
            ptrs = (C.c_void_p * len(parts))(*[p.data_ptr() for p in parts])
            ns = (C.c_int64 * len(parts))(*[p.shape[0] for p in parts])
            wid = lib.rb_pack_f32_q8_0_device(ptrs, ns, len(parts), parts[0].shape[1])
            _check(wid, "rocket_pack", 0, parts[0].shape[1], sum(p.shape[0] for p in parts))
            return WeightId(int(wid))

        def ones(n):
            return torch.ones(n, device=dev)

        self.gated = I % 64 == 0  # fused gate|up + silu_mul epilogue

        def pack_gu(gate, up):
            return pack_gated_q8_0(gate, up) if self.gated else pack_dev(
                [m for e in range(E) for m in (gate[e * I:(e + 1) * I], up[e * I:(e + 1) * I])])

        self.layers = []
        for li in range(cfg.layers):
            if host_weights is not None:
                W = host_weights["layers"][li]
                t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
                qkv = pack_dev([t(W["wq"]), t(W["wk"]), t(W["wv"])])
                o = pack_dev([t(W["wo"])])
                router = pack_dev([t(W["router"])])
                gu = pack_gu(torch.cat([t(gate) for gate, _, _ in W["experts"]]),
                             torch.cat([t(up) for _, up, _ in W["experts"]]))
                down = pack_dev([t(dn) for _, _, dn in W["experts"]])
                norms = {k: t(W[k]) for k in ("in_norm", "post_norm", "q_norm", "k_norm")}
            else:
                qkv = pack_dev([randn(nh * d, h), randn(nkv * d, h), randn(nkv * d, h)])
                o = pack_dev([randn(h, nh * d)])
                router = pack_dev([randn(E, h)])
                # experts: gate and up blocks stacked along N, then down blocks
                gate, up = randn(E * I, h), randn(E * I, h)
                gu = pack_gu(gate, up)
                del gate, up
                big = randn(E * h, I)
                down = pack_dev([big])
                del big
                norms = {"in_norm": ones(h), "post_norm": ones(h), "q_norm": ones(d), "k_norm": ones(d)}
            self.layers.append({"qkv": qkv, "o": o, "router": router, "gu": gu, "down": down, **norms})
        if host_weights is not None:
            self.final_norm = torch.from_numpy(host_weights["final_norm"]).to(dev).float()
            self.embed = torch.from_numpy(host_weights["embed"]).to(dev).half().contiguous()
        else:
            self.final_norm = ones(h)
            self.embed = (torch.randn(cfg.vocab, h, generator=g, device=dev) * 0.02).half().contiguous()
        cos, sin = rope_tables(seq, d, cfg.theta)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        torch.cuda.synchronize()
        f16 = torch.float16
        self.max_rows = int(lib.rb_moe_max_rows(T, cfg.top_k, E))
        ws_bytes = int(lib.rb_moe_workspace_bytes(T, cfg.top_k, E))
        self.ids_in = torch.zeros(T, dtype=torch.int32, device=dev)  # input token ids
        self.x = torch.empty(T, h, dtype=torch.float32, device=dev)
        self.h = torch.empty(T, h, dtype=f16, device=dev)
        self.qkv = torch.empty(T, (nh + 2 * nkv) * d, dtype=f16, device=dev)
        self.attn = torch.empty(T, nh * d, dtype=f16, device=dev)
        self.o = torch.empty(T, h, dtype=f16, device=dev)
        self.logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        self.ids = torch.empty(T, cfg.top_k, dtype=torch.int32, device=dev)
        self.wts = torch.empty(T, cfg.top_k, dtype=torch.float32, device=dev)
        self.ws = torch.empty((ws_bytes + 3) // 4, dtype=torch.int32, device=dev)
        self.xp = torch.empty(self.max_rows, h, dtype=f16, device=dev)
        self.gup = None if self.gated else torch.empty(self.max_rows, 2 * I, dtype=f16, device=dev)
        self.actp = torch.empty(self.max_rows, I, dtype=f16, device=dev)
        self.yp = torch.empty(self.max_rows, h, dtype=f16, device=dev)
        self.out = torch.empty(T, h, dtype=f16, device=dev)
        self.routing = []  # per layer (ids, wts) copies when record_routing
        self.graph = None

    # ------------------------------------------------------------------ forward
    def _layer(self, L: dict, stream=None, record_routing: bool = False):
        """One decoder layer on the residual stream self.x, in place (both
        residual adds included)."""
        cfg, lib, T = self.cfg, _lib.load(), self.T
        st = _stream_ptr(stream)
        h, d, nh, nkv, E, I, k = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.inter, cfg.top_k
        ld = (nh + 2 * nkv) * d
        qkv_p, xp, ws = _dev_ptr(self.qkv), _dev_ptr(self.x), _dev_ptr(self.ws)
        _check(lib.rb_add_rms_norm(xp, None, _dev_ptr(L["in_norm"]), cfg.eps, _dev_ptr(self.h), T, h, st),
               "add_rms_norm")
        matmul(self.h, L["qkv"], out=self.qkv, stream=stream)
        _check(lib.rb_qk_norm_rope(qkv_p, ld, T, nh, nkv, d, _dev_ptr(L["q_norm"]), _dev_ptr(L["k_norm"]),
                                   cfg.eps, _dev_ptr(self.cos), _dev_ptr(self.sin), self.seq, st),
               "qk_norm_rope")
        _check(lib.rb_attention_batched(qkv_p, ld, qkv_p + nh * d * 2, ld, qkv_p + (nh + nkv) * d * 2, ld,
                                        _dev_ptr(self.attn), nh * d, DTYPE_F16, self.batch, self.seq, self.seq,
                                        nh, nkv, d, 1.0 / math.sqrt(d), 0.0, MASK_CAUSAL, -1, 0, 0, st),
               "rocket_flash_attn", self.seq, self.seq, d)
        matmul(self.attn, L["o"], out=self.o, stream=stream)
        _check(lib.rb_add_rms_norm(xp, _dev_ptr(self.o), _dev_ptr(L["post_norm"]), cfg.eps, _dev_ptr(self.h),
                                   T, h, st), "add_rms_norm")
        matmul(self.h, L["router"], out=self.logits, stream=stream)
        _check(lib.rb_moe_route(_dev_ptr(self.logits), T, E, k, 1, _dev_ptr(self.ids), _dev_ptr(self.wts), st),
               "moe_route")
        if record_routing:
            self.routing.append((self.ids.clone(), self.wts.clone()))
        _check(lib.rb_moe_dispatch(_dev_ptr(self.ids), T, k, E, _dev_ptr(self.h), h, ws, _dev_ptr(self.xp), st),
               "moe_dispatch")
        if self.gated:  # silu(gate x) * (up x) straight from the grouped GEMM
            _check(lib.rb_matmul_grouped(L["gu"].id, E, _dev_ptr(self.xp), self.max_rows, ws, T, k,
                                         _dev_ptr(self.actp), DTYPE_F16, st), "matmul_grouped")
        else:
            _check(lib.rb_matmul_grouped(L["gu"].id, E, _dev_ptr(self.xp), self.max_rows, ws, T, k,
                                         _dev_ptr(self.gup), DTYPE_F16, st), "matmul_grouped")
            _check(lib.rb_silu_mul_halves(_dev_ptr(self.gup), self.max_rows, I, _dev_ptr(self.actp), st),
                   "silu_mul")
        _check(lib.rb_matmul_grouped(L["down"].id, E, _dev_ptr(self.actp), self.max_rows, ws, T, k,
                                     _dev_ptr(self.yp), DTYPE_F16, st), "matmul_grouped")
        _check(lib.rb_moe_combine(xp, _dev_ptr(self.yp), h, _dev_ptr(self.ids), _dev_ptr(self.wts), ws, T, k, E,
                                  st), "moe_combine")

    def embed_device(self, stream=None):
        """self.x = the f32 embedding rows of self.ids_in (the residual stream's start)."""
        cfg, lib = self.cfg, _lib.load()
        _check(lib.rb_embed_gather(_dev_ptr(self.ids_in), self.T, _dev_ptr(self.embed), cfg.vocab, cfg.hidden,
                                   _dev_ptr(self.x), _stream_ptr(stream)), "embed_gather")
        return self.x

    def forward_device(self, stream=None, record_routing: bool = False):
        """One forward over self.ids_in (int32 [T]) into self.out (f16, final-normed)."""
        cfg, lib = self.cfg, _lib.load()
        self.embed_device(stream)
        self.routing = []
        for L in self.layers:
            self._layer(L, stream, record_routing)
        _check(lib.rb_add_rms_norm(_dev_ptr(self.x), None, _dev_ptr(self.final_norm), cfg.eps, _dev_ptr(self.out),
                                   self.T, cfg.hidden, _stream_ptr(stream)), "add_rms_norm")
        return self.out

    def layer_step(self, li: int, stream=None):
        """Layer li alone on self.x (its output residual stream left in self.x;
        the layer's routing in self.ids / self.wts): a per-layer view of
        forward_device for checking each layer from the device's own input."""
        self._layer(self.layers[li], stream)
        return self.x

    def capture(self):
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

    def prefill_host(self, ids_host, out_host=None):
        """End-to-end call: host token ids [T] int32 in, final-normed f16 hidden states out."""
        import torch
        self.ids_in.copy_(ids_host, non_blocking=True)
        self.run()
        if out_host is None:
            out_host = torch.empty(self.T, self.cfg.hidden, dtype=torch.float16, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return out_host
