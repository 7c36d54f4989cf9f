"""SigLIP-style W8A8 vision tower on librocket_b200 (BASELINE config #4).

A synthetic pre-LayerNorm encoder: per layer
    h = layer_norm_1(x)
    q|k|v = h · Wqkv^T            (one fused W8A8 matmul, matmul_qat ext.rs:1245-1373)
    x += attention(q, k, v) · Wo^T  (bidirectional, 16 heads x 72, attention_window(-1)
                                   as the reference's vision tower calls it, ext.rs:1907-1950)
    h = layer_norm_2(x)
    x += gelu_tanh(h · W1^T) · W2^T  (gelu_tanh of host.rs:15-18)
then the final (post) LayerNorm of every patch. Every projection is W8A8:
int8 per-output-channel weight codes (the fp16 weights quantised on the device
by rb_pack_f32_w8a8_device, the form pack_qat takes, ext.rs:1382-1425) and
dynamic per-token int8 activation codes with the f32 epilogue of
matmul_qat. Linear layers carry no bias (the reference's W8A8 op has none).

Every op is a librocket_b200 kernel launched through the C ABI; torch only
allocates device buffers, generates the synthetic weights and captures the
call sequence into a CUDA graph. The residual stream is f32; matmul
inputs/outputs are f16. Images are independent, so data parallelism shards
them over GPUs with no collective.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

from . import _lib
from . import _check, _dev_ptr, _stream_ptr, matmul, pack_w8a8_float, set_weight_activation
from ._lib import DTYPE_F16, MASK_NONE


@dataclass(frozen=True)
class SiglipConfig:
    layers: int = 27
    hidden: int = 1152
    heads: int = 16
    head_dim: int = 72
    inter: int = 4304
    eps: float = 1e-6
    patches: int = 2394

    @property
    def linear_params_per_layer(self) -> int:
        h = self.hidden
        return 3 * h * self.heads * self.head_dim + self.heads * self.head_dim * h + 2 * h * self.inter

    def ops_per_patch(self) -> tuple[float, float]:
        """(int8 linear ops, attention FLOPs) per patch: 2·params and 4·S·D·H, per layer."""
        lin = self.layers * 2.0 * self.linear_params_per_layer
        att = self.layers * 4.0 * self.patches * self.head_dim * self.heads
        return lin, att


class SiglipTower:
    """Resident random-init tower (W8A8 linears) + preallocated activations for
    `images` images of cfg.patches patch embeddings on the current CUDA device."""

    def __init__(self, cfg: SiglipConfig, images: int, seed: int = 0, host_weights: dict | None = None):
        import torch
        self.cfg, self.images = cfg, images
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        T = images * cfg.patches
        self.T = T
        g = torch.Generator(device=dev).manual_seed(seed)
        h, inter = cfg.hidden, cfg.inter
        hq = cfg.heads * cfg.head_dim

        def randn16(*shape):
            # fp16 weights ~ N(0, 0.02), widened for the device quantiser
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * 0.02).half().float()

        def pack(w):
            return pack_w8a8_float(w)

        def ln_pair(n):
            return (torch.ones(n, device=dev), torch.zeros(n, device=dev))

        self.layers = []
        for li in range(cfg.layers):
            if host_weights is not None:
                W = {k: torch.from_numpy(v).to(dev) for k, v in host_weights["layers"][li].items()}
            else:
                g1, b1 = ln_pair(h)
                g2, b2 = ln_pair(h)
                W = {"wq": randn16(hq, h), "wk": randn16(hq, h), "wv": randn16(hq, h), "wo": randn16(h, hq),
                     "w1": randn16(inter, h), "w2": randn16(h, inter),
                     "ln1_g": g1, "ln1_b": b1, "ln2_g": g2, "ln2_b": b2}
            fc1 = pack(W["w1"])
            set_weight_activation(fc1, "gelu_tanh")  # gelu_tanh fused into the fc1 epilogue
            self.layers.append({
                "qkv": pack(torch.cat([W["wq"], W["wk"], W["wv"]], 0)),
                "o": pack(W["wo"]), "fc1": fc1, "fc2": pack(W["w2"]),
                "ln1_g": W["ln1_g"].float().contiguous(), "ln1_b": W["ln1_b"].float().contiguous(),
                "ln2_g": W["ln2_g"].float().contiguous(), "ln2_b": W["ln2_b"].float().contiguous(),
            })
            del W
        if host_weights is not None:
            self.post_g = torch.from_numpy(host_weights["post_g"]).to(dev).float().contiguous()
            self.post_b = torch.from_numpy(host_weights["post_b"]).to(dev).float().contiguous()
        else:
            self.post_g, self.post_b = ln_pair(h)
        torch.cuda.synchronize()
        f16 = torch.float16
        self.patches = torch.empty(T, h, dtype=torch.float32, device=dev)  # input patch embeddings
        self.x = torch.empty(T, h, dtype=torch.float32, device=dev)
        self.h = torch.empty(T, h, dtype=f16, device=dev)
        # pre-LN rows quantised in the LayerNorm kernel for the W8A8 qkv / fc1 matmuls
        self.hc = torch.empty(T, h, dtype=torch.int8, device=dev)
        self.hs = torch.empty(T, dtype=torch.float32, device=dev)
        self.qkv = torch.empty(T, 3 * hq, dtype=f16, device=dev)
        self.attn = torch.empty(T, hq, dtype=f16, device=dev)
        self.o = torch.empty(T, h, dtype=f16, device=dev)
        self.f = torch.empty(T, inter, dtype=f16, device=dev)
        self.d = torch.empty(T, h, dtype=f16, device=dev)
        self.out = torch.empty(T, h, dtype=f16, device=dev)
        self.graph = None

    # ------------------------------------------------------------------ forward
    def _rows(self, img0: int, n_img: int | None):
        S = self.cfg.patches
        n_img = self.images - img0 if n_img is None else n_img
        r0, T = img0 * S, n_img * S
        return n_img, T, (lambda t: t[r0:r0 + T])

    def _layer(self, L: dict, delta, stream=None, img0: int = 0, n_img: int | None = None):
        """One encoder layer on the residual stream self.x (rows of images
        [img0, img0 + n_img)): `delta` (a device pointer or None) is the previous
        layer's pending MLP output, folded into this layer's first residual-add
        + LayerNorm. Returns this layer's pending MLP output pointer."""
        cfg, lib = self.cfg, _lib.load()
        st = _stream_ptr(stream)
        h, hq, S = cfg.hidden, cfg.heads * cfg.head_dim, cfg.patches
        ld = 3 * hq
        n_img, T, rows = self._rows(img0, n_img)
        x, hc, hs, qkv, attn, o, f, d = (rows(t) for t in (self.x, self.hc, self.hs, self.qkv, self.attn,
                                                            self.o, self.f, self.d))
        qkv_p = _dev_ptr(qkv)
        _check(lib.rb_add_layer_norm_quant(_dev_ptr(x), delta, _dev_ptr(L["ln1_g"]), _dev_ptr(L["ln1_b"]),
                                           cfg.eps, _dev_ptr(hc), _dev_ptr(hs), T, h, st),
               "add_layer_norm_quant")
        _check(lib.rb_matmul_w8a8_codes(L["qkv"].id, _dev_ptr(hc), _dev_ptr(hs), T, h, qkv_p,
                                        DTYPE_F16, st), "rocket_matmul", T, h, 3 * hq)
        _check(lib.rb_attention_batched(qkv_p, ld, qkv_p + hq * 2, ld, qkv_p + 2 * hq * 2, ld,
                                        _dev_ptr(attn), hq, DTYPE_F16, n_img, S, S,
                                        cfg.heads, cfg.heads, cfg.head_dim, 1.0 / math.sqrt(cfg.head_dim),
                                        0.0, MASK_NONE, -1, 0, 0, st),
               "rocket_flash_attn", S, S, cfg.head_dim)
        matmul(attn, L["o"], out=o, stream=stream)
        _check(lib.rb_add_layer_norm_quant(_dev_ptr(x), _dev_ptr(o), _dev_ptr(L["ln2_g"]),
                                           _dev_ptr(L["ln2_b"]), cfg.eps, _dev_ptr(hc), _dev_ptr(hs),
                                           T, h, st), "add_layer_norm_quant")
        _check(lib.rb_matmul_w8a8_codes(L["fc1"].id, _dev_ptr(hc), _dev_ptr(hs), T, h,
                                        _dev_ptr(f), DTYPE_F16, st), "rocket_matmul", T, h, cfg.inter)
        # (gelu_tanh(h W1^T) is fused into the fc1 epilogue)
        matmul(f, L["fc2"], out=d, stream=stream)
        return _dev_ptr(d)

    def forward_device(self, stream=None, img0: int = 0, n_img: int | None = None):
        """One forward over self.patches (f32 [T, hidden]) into self.out (f16 [T, hidden]);
        img0 / n_img restrict it to the images [img0, img0 + n_img) (their rows
        of every buffer; images are independent)."""
        import torch
        cfg, lib = self.cfg, _lib.load()
        st = _stream_ptr(stream)
        n_img, T, rows = self._rows(img0, n_img)
        x, out = rows(self.x), rows(self.out)
        # the residual stream starts as the input (x is rewritten in place each layer)
        if stream is None:
            x.copy_(rows(self.patches))
        else:
            with torch.cuda.stream(stream):
                x.copy_(rows(self.patches))
        delta = None
        for L in self.layers:
            delta = self._layer(L, delta, stream, img0, n_img)
        _check(lib.rb_add_layer_norm(_dev_ptr(x), delta, _dev_ptr(self.post_g), _dev_ptr(self.post_b), cfg.eps,
                                     _dev_ptr(out), T, cfg.hidden, st), "add_layer_norm")
        return self.out

    def layer_step(self, li: int, stream=None):
        """Layer li alone on self.x (all images), leaving its output residual
        stream in self.x (the pending MLP output folded in; self.out is
        scratch): a per-layer view of forward_device for checking each layer
        from the device's own input."""
        cfg, lib = self.cfg, _lib.load()
        delta = self._layer(self.layers[li], None, stream)
        _check(lib.rb_add_layer_norm(_dev_ptr(self.x), delta, _dev_ptr(self.post_g), _dev_ptr(self.post_b),
                                     cfg.eps, _dev_ptr(self.out), self.T, cfg.hidden, _stream_ptr(stream)),
               "add_layer_norm")
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

    def encode_host(self, patches_host, out_host=None, overlap: bool = False):
        """End-to-end call: host patch embeddings [images*patches, hidden] f32 in,
        host f16 patch states out. overlap=True (two or more images, page-locked
        host buffers) runs the tower as two halves of the images, each from its
        own captured CUDA graph: the second half's input copies in while the
        first half computes, and the first half's output copies out while the
        second computes. Results then equal the whole-batch forward up to the
        f32 summation order of attention."""
        import torch
        if out_host is None:
            out_host = torch.empty(self.T, self.cfg.hidden, dtype=torch.float16, pin_memory=True)
        if not (overlap and self.images >= 2):
            self.patches.copy_(patches_host, non_blocking=True)
            self.run()
            out_host.copy_(self.out, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return out_host
        half = self.images // 2
        if getattr(self, "half_graphs", None) is None:
            graphs = []
            for i0, n in ((0, half), (half, self.images - half)):
                self.forward_device(img0=i0, n_img=n)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    self.forward_device(img0=i0, n_img=n)
                graphs.append(g)
            self.half_graphs = graphs
            self.copy_in, self.copy_out = torch.cuda.Stream(), torch.cuda.Stream()
        r = half * self.cfg.patches
        cur = torch.cuda.current_stream()
        self.copy_in.wait_stream(cur)
        with torch.cuda.stream(self.copy_in):
            self.patches[:r].copy_(patches_host[:r], non_blocking=True)
            in_a = torch.cuda.current_stream().record_event()
            self.patches[r:].copy_(patches_host[r:], non_blocking=True)
            in_b = torch.cuda.current_stream().record_event()
        cur.wait_event(in_a)
        self.half_graphs[0].replay()
        done_a = cur.record_event()
        self.copy_out.wait_event(done_a)
        with torch.cuda.stream(self.copy_out):
            out_host[:r].copy_(self.out[:r], non_blocking=True)
        cur.wait_event(in_b)
        self.half_graphs[1].replay()
        out_host[r:].copy_(self.out[r:], non_blocking=True)
        cur.synchronize()
        self.copy_out.synchronize()
        return out_host
