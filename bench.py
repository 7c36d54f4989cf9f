"""bench.py — throughput of the offloaded ops on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload qwen3|attn|q8gemm|w8a8|siglip|moe] [--impl b200|reference]

BASELINE.json's metric has three items: "Q8_0/W8A8 GEMM TFLOP/s; GQA attn
TFLOP/s; Qwen3-Emb-0.6B prefill tok/s". The default line is the model item,
config #3, and it carries sub-records (key "sub"), each with its own
ms_per_step, roofline and e2e: config #4's W8A8 tower data-parallel over the
same N GPUs (every N), config #5's MoE expert-parallel over them (N >= 2,
with its all-to-all time and share), and at N = 1 one record per single-op
item (config #1 Q8_0 GEMM, config #2 attention, config #4's W8A8
projections, group-wise int8), each timed alone.

Workloads (synthetic seeded data of the named shapes):
  qwen3   config #3 (default): Qwen3-Embedding-0.6B-architecture forward, 28
          layers, 64 sequences x 512 tokens, bidirectional, random-init Q8_0
          linears; data-parallel over sequences (64/N per GPU, global batch
          fixed: strong scaling). Metric: tokens/s.
  q8gemm  config #1: f32 [512, 1024] x Q8_0 [3072, 1024]^T -> f32 [512, 3072].
  attn    config #2: GQA attention, 3633 tokens, 16 q / 8 kv heads x 128, fp16,
          RoPE (theta 1e6) pre-applied; one step = one causal + one
          bidirectional call. Metric: attention TFLOP/s (algorithmic FLOPs:
          4*S*S*D*H bidirectional, 4*D*H*S(S+1)/2 causal).
  w8a8    config #4's four projection GEMMs (qkv 3456, o 1152, fc1 4304,
          fc2 1152 <- 4304) over one 16 x 2394-patch batch, W8A8, with the
          tower's fp16 activations in and out (dynamic per-token int8
          quantisation of the f16 input inside the step).
  siglip  config #4: the SigLIP-style W8A8 tower, 16 images, DP over images.
  moe     config #5: Qwen3-30B-A3B-style MoE prefill (EP over N GPUs).

Timing: W untimed warm-up steps, then exactly K steps timed with CUDA events on
the launching stream, an L2 flush (a 256 MiB write) between timed steps, a
barrier + synchronize on both sides, max over ranks. The single ops do not
shard: with N > 1 each rank runs an independent replica and `value` is the
aggregate over ranks. The `e2e` figure goes through the public host entry
points (rb_*_host, the models' embed_host / encode_host / prefill_host) with
pinned host buffers, so host<->device copies are inside its timed region.

`--impl reference` times the reference algorithm on the host cores instead:
the CPU restatement of the reference's `--device cpu` path (oracle/, OpenMP
on every host core), on a bounded sample of the same workload; rank 0 alone
runs under torchrun.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# Committed ncu summary of each workload's dominant kernel (profiles/).
PROFILES = {
    "attn": "attn_kernel_gqa_s3633_ncu.md",
    "q8gemm": "gemm_pair_kernel_q8_0_config1_ncu.md",
    "w8a8": "gemm_pair_kernel_w8a8_8192x4304x1152_ncu.md",
    "w8a8g": "gemm_i8g_kernel_g128_config4_ncu.md",
    "qwen3": "gemm_pair_kernel_q8_0_8192x6144x1024_ncu.md",
    "siglip": "gemm_pair_kernel_w8a8_8192x4304x1152_ncu.md",
    "moe": "gemm_pair_kernel_moe_grouped_ncu.md",
}


def profile_traffic(workload):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary."""
    if workload not in PROFILES:
        return None
    p = ROOT / "profiles" / PROFILES[workload]
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks and throttle reasons (NVML, the counters nvidia-smi
    reports) every few milliseconds while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, torch_device_index, period_s=0.005):
        self.idx = torch_device_index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self.handle = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.idx)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.idx)

    def _run(self):
        import pynvml
        while not self._stop.is_set():
            try:
                self.samples.append(pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        try:
            import pynvml
            self.handle = self._open()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.handle = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.handle is not None:
            self.t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- workloads
def rope_inplace(x, n_heads, d, theta=1e6):
    """Rotate-half RoPE (util/rope.rs:15-75) on a [S, H*D] tensor, positions 0..S-1."""
    import torch
    s = x.shape[0]
    half = d // 2
    inv = torch.tensor([1.0 / theta ** (2.0 * i / d) for i in range(half)], dtype=torch.float64).float()
    pos = torch.arange(s, dtype=torch.float32)
    ang = pos[:, None] * inv[None, :]
    cos, sin = ang.cos().to(x.device), ang.sin().to(x.device)
    xv = x.float().view(s, n_heads, d)
    x1, x2 = xv[..., :half], xv[..., half:]
    o1 = x1 * cos[:, None, :] - x2 * sin[:, None, :]
    o2 = x2 * cos[:, None, :] + x1 * sin[:, None, :]
    return torch.cat([o1, o2], -1).reshape(s, n_heads * d).to(x.dtype)


class AttnWorkload:
    name = "attn"
    metric = "GQA attention TFLOP/s (config #2: S=3633, 16q/8kv x 128, causal + bidirectional)"
    unit = "TFLOP/s"
    S, H, KV, D = 3633, 16, 8, 128

    def __init__(self, dev, seed):
        import torch
        import burn_rocket_b200 as rb
        self.rb = rb
        g = torch.Generator(device="cpu").manual_seed(seed)
        S, H, KV, D = self.S, self.H, self.KV, self.D
        q = torch.randn(S, H * D, generator=g)
        k = torch.randn(S, KV * D, generator=g)
        v = torch.randn(S, KV * D, generator=g)
        self.q = rope_inplace(q, H, D).half().to(dev)
        self.k = rope_inplace(k, KV, D).half().to(dev)
        self.v = v.half().to(dev)
        self.out_c = torch.empty_like(self.q)
        self.out_b = torch.empty_like(self.q)
        self.scale = 1.0 / math.sqrt(D)
        self.flops_b = 4.0 * S * S * D * H
        self.flops_c = 4.0 * D * H * S * (S + 1) / 2
        self.flops = self.flops_b + self.flops_c
        # pinned host copies for the end-to-end leg
        self.hq = self.q.cpu().pin_memory()
        self.hk = self.k.cpu().pin_memory()
        self.hv = self.v.cpu().pin_memory()
        self.hout = torch.empty_like(self.hq).pin_memory()

    def step(self):
        rb = self.rb
        rb.attention(self.q, self.k, self.v, self.H, self.KV, self.D, self.scale, None, True, out=self.out_c)
        rb.attention(self.q, self.k, self.v, self.H, self.KV, self.D, self.scale, None, False, out=self.out_b)

    def kernel_launches(self):
        return [("attn_kernel causal", self.flops_c), ("attn_kernel bidirectional", self.flops_b)]

    def beside(self, stream, peak):
        """Reported beside config #2: config #4's head_dim-72 attention (16
        images x 2394 patches, 16 heads x 72, bidirectional; q/k/v strided
        inside the tower's [rows, 3 x 1152] qkv buffer, 265 MB: larger than
        L2), one rb_attention_batched call per step, 20 steps back to back."""
        import torch
        import burn_rocket_b200._lib as L
        n_img, T, h, hd = 16, 2394, 16, 72
        hq = h * hd
        g = torch.Generator(device="cpu").manual_seed(7)
        qkv = torch.randn(n_img * T, 3 * hq, generator=g).half().to(self.q.device)
        att = torch.empty(n_img * T, hq, dtype=torch.half, device=self.q.device)
        p0, lib = qkv.data_ptr(), L.load()

        def call():
            rc = lib.rb_attention_batched(p0, 3 * hq, p0 + hq * 2, 3 * hq, p0 + 2 * hq * 2, 3 * hq, att.data_ptr(), hq,
                                          L.DTYPE_F16, n_img, T, T, h, h, hd, 1.0 / math.sqrt(hd), 0.0,
                                          L.MASK_NONE, -1, 0, 0, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(L.last_error())
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        steps = 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        a.record(stream)
        for _ in range(steps):
            call()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        tflops = 4.0 * T * T * hd * h * n_img / (ms / 1e3) / 1e12
        return {"siglip_hd72": {"what": "config #4 tower attention, 16 x 2394 patches, 16 heads x 72, bidirectional",
                                "ms_per_call": round(ms, 4), "tflops": round(tflops, 1),
                                "frac_of_burst": round(tflops / peak, 4)}}

    def e2e_step(self):
        import burn_rocket_b200._lib as L
        lib = L.load()
        for mode in (L.MASK_CAUSAL, L.MASK_NONE):
            rc = lib.rb_attention_host(self.hq.data_ptr(), self.hk.data_ptr(), self.hv.data_ptr(),
                                       self.hout.data_ptr(), L.DTYPE_F16, self.S, self.S, self.H, self.KV, self.D,
                                       self.scale, 0.0, mode, -1, 0, 0)
            if rc != 0:
                raise RuntimeError(L.last_error())
        return (2 * (self.hq.numel() + self.hk.numel() + self.hv.numel()) * 2, 2 * self.hout.numel() * 2)

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        """Reference CPU algorithm on 1 of the 8 KV groups (2 of 16 heads), causal + bidirectional."""
        S, D = AttnWorkload.S, AttnWorkload.D
        rng = np.random.default_rng(seed)
        q = rng.standard_normal((S, 2 * D)).astype(np.float32)
        k = rng.standard_normal((S, D)).astype(np.float32)
        v = rng.standard_normal((S, D)).astype(np.float32)
        flops = 4.0 * S * S * D * 2 + 4.0 * D * 2 * S * (S + 1) / 2
        t0 = time.perf_counter()
        for _ in range(timed_repeats):
            orc.attention_cpu(q, k, v, 2, 1, D, 1.0 / math.sqrt(D), True)
            orc.attention_cpu(q, k, v, 2, 1, D, 1.0 / math.sqrt(D), False)
        dt = (time.perf_counter() - t0) / timed_repeats
        return flops / dt / 1e12, "1 of 8 KV groups (2 of 16 q heads), full 3633 tokens, causal + bidirectional"


class Q8GemmWorkload:
    name = "q8gemm"
    metric = "Q8_0 GEMM TFLOP/s (config #1: f32 [512,1024] x Q8_0 [3072,1024]^T)"
    unit = "TFLOP/s"
    M, K, N = 512, 1024, 3072
    X_DTYPE = "f32"

    def __init__(self, dev, seed):
        import torch
        import burn_rocket_b200 as rb
        self.rb = rb
        if (self.M, self.N, self.K) != (512, 3072, 1024):
            self.metric = f"Q8_0 GEMM TFLOP/s ([{self.M},{self.K}] {self.X_DTYPE} x Q8_0 [{self.N},{self.K}]^T)"
        rng = np.random.default_rng(seed)
        a = rng.standard_normal((self.M, self.K)).astype(np.float32)
        w = (rng.standard_normal((self.N, self.K)) * 0.02).astype(np.float32)
        self.wid = rb.pack_q8_0(w)  # device Q8_0 encoder
        xdt = torch.float32 if self.X_DTYPE == "f32" else torch.float16
        self.x = torch.from_numpy(a).to(dev).to(xdt)
        self.y = torch.empty(self.M, self.N, dtype=xdt, device=dev)
        self.flops = 2.0 * self.M * self.N * self.K
        self.weight_bytes = self.N * self.K * (1 + 2 / 32)  # Q8_0 codes + f16 block scales
        self.hx = self.x.cpu().pin_memory()
        self.hy = torch.empty(self.M, self.N, dtype=xdt).pin_memory()

    def step(self):
        self.rb.matmul(self.x, self.wid, out=self.y)

    def kernel_launches(self):
        return [("q8_0 gemm (+ f32->f16 cast)", self.flops)]

    def e2e_step(self):
        import burn_rocket_b200._lib as L
        dt = L.DTYPE_F32 if self.X_DTYPE == "f32" else L.DTYPE_F16
        rc = L.load().rb_matmul_host(self.wid.id, self.hx.data_ptr(), dt, self.M, self.K,
                                     self.hy.data_ptr(), dt)
        if rc != 0:
            raise RuntimeError(L.last_error())
        return (self.hx.numel() * self.hx.element_size(), self.hy.numel() * self.hy.element_size())

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=3):
        M, K, N = Q8GemmWorkload.M, Q8GemmWorkload.K, Q8GemmWorkload.N
        rng = np.random.default_rng(seed)
        a = rng.standard_normal((M, K)).astype(np.float32)
        codes, scales = orc.q8_0_quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        scratch = np.empty((N, K), np.float32)
        orc.q8_0_matmul_cpu(a, codes, scales, scratch)
        t0 = time.perf_counter()
        for _ in range(timed_repeats):
            orc.q8_0_matmul_cpu(a, codes, scales, scratch)
        dt = (time.perf_counter() - t0) / timed_repeats
        return 2.0 * M * N * K / dt / 1e12, "full config #1 call (dequantise + f32 GEMM)"


class W8A8Workload:
    name = "w8a8"
    metric = "W8A8 GEMM TOP/s (config #4 projections qkv/o/fc1/fc2 over 16 x 2394 patches, f16 in/out)"
    unit = "TOP/s"
    M = M_CONFIG = 16 * 2394
    SHAPES = SHAPES_CONFIG = [(3456, 1152), (1152, 1152), (4304, 1152), (1152, 4304)]  # (N, K)
    X_DTYPE = "f16"  # config #3's tower is fp16: f16 activations in, f16 out

    def __init__(self, dev, seed):
        import torch
        import burn_rocket_b200 as rb
        self.rb = rb
        rng = np.random.default_rng(seed)
        if (self.M, self.SHAPES) != (W8A8Workload.M_CONFIG, W8A8Workload.SHAPES_CONFIG):
            self.metric = "W8A8 GEMM TOP/s (" + ", ".join(f"[{self.M},{k}] {self.X_DTYPE} x s8 [{n},{k}]^T"
                                                          for n, k in self.SHAPES) + ")"
        xdt = torch.float32 if self.X_DTYPE == "f32" else torch.float16
        self.ws, self.xs, self.ys = [], [], []
        for n, k in self.SHAPES:
            codes = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
            scale = (rng.random(n).astype(np.float32) * 1e-3 + 1e-4)
            self.ws.append(rb.pack_qat(codes, scale, n, k))
            self.xs.append(torch.randn(self.M, k, device=dev).to(xdt))
            self.ys.append(torch.empty(self.M, n, dtype=xdt, device=dev))
        self.flops = sum(2.0 * self.M * n * k for n, k in self.SHAPES)
        self.weight_bytes = sum(n * k + 4 * n for n, k in self.SHAPES)
        self.hx = [x.cpu().pin_memory() for x in self.xs]
        self.hy = [y.cpu().pin_memory() for y in self.ys]

    def step(self):
        for w, x, y in zip(self.ws, self.xs, self.ys):
            self.rb.matmul(x, w, out=y)

    def kernel_launches(self):
        return [(f"w8a8 gemm N={n} K={k} (+ row quantiser)", 2.0 * self.M * n * k) for n, k in self.SHAPES]

    def e2e_step(self):
        import burn_rocket_b200._lib as L
        h2d = d2h = 0
        dt = L.DTYPE_F32 if self.X_DTYPE == "f32" else L.DTYPE_F16
        for (n, k), w, hx, hy in zip(self.SHAPES, self.ws, self.hx, self.hy):
            rc = L.load().rb_matmul_host(w.id, hx.data_ptr(), dt, self.M, k, hy.data_ptr(), dt)
            if rc != 0:
                raise RuntimeError(L.last_error())
            h2d += hx.numel() * hx.element_size()
            d2h += hy.numel() * hy.element_size()
        return (h2d, d2h)

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        rng = np.random.default_rng(seed)
        rows = 512
        flops = 0.0
        t = 0.0
        for n, k in W8A8Workload.SHAPES:
            x = rng.standard_normal((rows, k)).astype(np.float32)
            codes = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
            s = np.full(n, 1e-3, np.float32)
            t0 = time.perf_counter()
            orc.w8a8_matmul(x, codes, s)
            t += time.perf_counter() - t0
            flops += 2.0 * rows * n * k
        return flops / t / 1e12, f"{rows} of {W8A8Workload.M} rows of each projection (quantise + int GEMM + epilogue)"


class W8A8GroupWorkload(W8A8Workload):
    """Config #4's projections with group-wise int8 weights and activations
    (rocket_pack_i8 / matmul_i8, g = 128, the Clef experts' group): the group
    quantiser and one GEMM with in-kernel group promotion per projection. The
    three projections with K = 1152 (qkv, o, fc1); fc2's K = 4304 is not a
    multiple of 32, which pack_i8 requires (ext.rs:948-953)."""
    name = "w8a8g"
    GROUP = 128
    SHAPES = [(3456, 1152), (1152, 1152), (4304, 1152)]  # (N, K)
    metric = "group-wise int8 GEMM TOP/s (g128; config #4 qkv/o/fc1 over 16 x 2394 patches, f16 in/out)"

    def __init__(self, dev, seed):
        import torch
        import burn_rocket_b200 as rb
        self.rb = rb
        rng = np.random.default_rng(seed)
        self.ws, self.xs, self.ys = [], [], []
        for n, k in self.SHAPES:
            w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
            self.ws.append(rb.pack_i8(w, self.GROUP))
            self.xs.append(torch.randn(self.M, k, device=dev).half())
            self.ys.append(torch.empty(self.M, n, dtype=torch.float16, device=dev))
        self.flops = sum(2.0 * self.M * n * k for n, k in self.SHAPES)
        self.weight_bytes = sum(n * k + 4 * n for n, k in self.SHAPES)
        self.hx = [x.cpu().pin_memory() for x in self.xs]
        self.hy = [y.cpu().pin_memory() for y in self.ys]

    def kernel_launches(self):
        return [(f"i8g gemm N={n} K={k} (+ group quantiser)", 2.0 * self.M * n * k) for n, k in self.SHAPES]

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        rng = np.random.default_rng(seed)
        rows, g = 256, W8A8GroupWorkload.GROUP
        flops, t = 0.0, 0.0
        for n, k in W8A8GroupWorkload.SHAPES:
            x = rng.standard_normal((rows, k)).astype(np.float32)
            wq, ws = orc.quantize_rows_groups((rng.standard_normal((n, k)) * 0.02).astype(np.float32), g)
            t0 = time.perf_counter()
            q, s = orc.quantize_rows_groups(x, g)
            orc.matmul_gw(q, s, wq, ws, g)
            t += time.perf_counter() - t0
            flops += 2.0 * rows * n * k
        return flops / t / 1e12, f"{rows} of {W8A8Workload.M} rows of each projection (group quantise + int GEMM + promotion)"


class Qwen3Workload:
    """Config #3: Qwen3-Embedding-0.6B-architecture forward, 64 sequences x 512
    tokens bidirectional, data-parallel over sequences (64/N per GPU)."""
    name = "qwen3"
    metric = "Qwen3-Emb-0.6B-arch prefill tok/s (config #3: 64 seq x 512 tok, bidirectional, Q8_0 linears)"
    unit = "tok/s"
    BATCH, SEQ = 64, 512

    def __init__(self, dev, seed, world=1, rank=0):
        import torch
        import burn_rocket_b200 as rb
        from burn_rocket_b200.qwen3 import Qwen3Config, Qwen3Embedding
        self.rb = rb
        self.cfg = Qwen3Config()
        if self.BATCH % world:
            raise SystemExit(f"--gpus {world} must divide the {self.BATCH}-sequence batch")
        self.local = self.BATCH // world
        # every rank holds the same random-init weights (seed 0); the token ids
        # of rank r are sequences [r*local, (r+1)*local) of the global batch.
        self.model = Qwen3Embedding(self.cfg, self.local, self.SEQ, seed=0)
        g = torch.Generator(device="cpu").manual_seed(seed)
        ids = torch.randint(0, self.cfg.vocab, (self.BATCH * self.SEQ,), generator=g, dtype=torch.int32)
        mine = ids[rank * self.local * self.SEQ:(rank + 1) * self.local * self.SEQ]
        self.model.ids.copy_(mine.to(dev))
        self.hids = mine.pin_memory()
        self.hout = torch.empty(self.local, self.cfg.hidden, dtype=torch.float32).pin_memory()
        self.units = self.local * self.SEQ  # tokens per step on this rank
        self.flops = self.cfg.flops_per_token(self.SEQ) * self.units

    def step(self):
        self.model.forward_device()

    def e2e_step(self):
        if self.model.graph is None:  # the public host call replays the model's CUDA graph
            self.model.capture()
        self.model.embed_host(self.hids, self.hout)
        return (self.hids.numel() * 4, self.hout.numel() * 4)

    def kernel_roofline(self):
        """Device time of the four Q8_0 GEMMs of one layer at the config shapes."""
        import torch
        m, L = self.model, self.model.layers[0]
        calls = [(m.h, L["qkv"], m.qkv), (m.attn, L["o"], m.o), (m.h, L["gu"], m.act), (m.act, L["down"], m.d)]
        flops = 0.0
        for x, w, y in calls:
            _, n, k = self.rb.weight_info(w)
            # a gated gate|up weight multiplies 2n rows for its n fused outputs
            flops += 2.0 * x.shape[0] * n * k * (2 if w is L["gu"] else 1)
        for _ in range(2):
            for x, w, y in calls:
                self.rb.matmul(x, w, out=y)
        reps = 5
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(reps):
            for x, w, y in calls:
                self.rb.matmul(x, w, out=y)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / reps
        return "q8_0 gemm_kernel (qkv, o, gate|up with fused silu_mul, down of one layer)", flops / (ms / 1e3) / 1e12, ms

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        """The reference CPU algorithm for one layer at 512 tokens (dequantise +
        f32 GEMM for the four projections, tiled f32 attention for one
        sequence), scaled to the 28-layer model."""
        from burn_rocket_b200.qwen3 import Qwen3Config
        cfg = Qwen3Config()
        rng = np.random.default_rng(seed)
        T, h = 512, cfg.hidden
        shapes = [((cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim, h), (h, cfg.heads * cfg.head_dim),
                  (2 * cfg.inter, h), (h, cfg.inter)]
        ws = [orc.q8_0_quantize((rng.standard_normal(sh) * 0.02).astype(np.float32)) for sh in shapes]
        xs = [rng.standard_normal((T, sh[1])).astype(np.float32) for sh in shapes]
        q = rng.standard_normal((T, cfg.heads * cfg.head_dim)).astype(np.float32)
        kv = rng.standard_normal((T, cfg.kv_heads * cfg.head_dim)).astype(np.float32)
        t0 = time.perf_counter()
        for _ in range(timed_repeats):
            for (codes, scales), x in zip(ws, xs):
                orc.q8_0_matmul_cpu(x, codes, scales)
            orc.attention_cpu(q, kv, kv, cfg.heads, cfg.kv_heads, cfg.head_dim, 1 / math.sqrt(cfg.head_dim), False)
        t_layer = (time.perf_counter() - t0) / timed_repeats
        return T / (t_layer * cfg.layers), "one layer (4 Q8_0 projections + attention) at 512 tokens, x28 layers"


class SiglipWorkload:
    """Config #4: SigLIP-style W8A8 vision tower, 16 images x 2394 patches,
    data-parallel over images (16/N per GPU)."""
    name = "siglip"
    metric = "SigLIP-style W8A8 tower patches/s (config #4: 16 images x 2394 patches, 27 layers)"
    unit = "patch/s"
    IMAGES = 16

    def __init__(self, dev, seed, world=1, rank=0):
        import torch
        import burn_rocket_b200 as rb
        from burn_rocket_b200.siglip import SiglipConfig, SiglipTower
        self.rb = rb
        self.cfg = SiglipConfig()
        if self.IMAGES % world:
            raise SystemExit(f"--gpus {world} must divide the {self.IMAGES}-image batch")
        self.local = self.IMAGES // world
        # identical random-init weights on every rank (seed 0); rank r encodes
        # images [r*local, (r+1)*local) of the global batch.
        self.model = SiglipTower(self.cfg, self.local, seed=0)
        S, h = self.cfg.patches, self.cfg.hidden
        g = torch.Generator(device="cpu").manual_seed(seed + rank)
        mine = torch.randn(self.local * S, h, generator=g)
        self.model.patches.copy_(mine.to(dev))
        self.hpatches = mine.pin_memory()
        self.hout = torch.empty(self.local * S, h, dtype=torch.float16).pin_memory()
        self.units = self.local * S  # patches per step on this rank
        lin, att = self.cfg.ops_per_patch()
        self.flops = (lin + att) * self.units

    def step(self):
        self.model.forward_device()

    def e2e_step(self):
        if self.model.graph is None:  # the public host call replays the model's CUDA graph
            self.model.capture()
        self.model.encode_host(self.hpatches, self.hout, overlap=True)
        return (self.hpatches.numel() * 4, self.hout.numel() * 2)

    def kernel_roofline(self):
        """Device time of the four W8A8 projections of one layer (row quantiser + int8 GEMM)."""
        import torch
        m, L = self.model, self.model.layers[0]
        calls = [(m.h, L["qkv"], m.qkv), (m.attn, L["o"], m.o), (m.h, L["fc1"], m.f), (m.f, L["fc2"], m.d)]
        ops = 0.0
        for x, w, y in calls:
            _, n, k = self.rb.weight_info(w)
            ops += 2.0 * x.shape[0] * n * k
        for _ in range(2):
            for x, w, y in calls:
                self.rb.matmul(x, w, out=y)
        reps = 5
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(reps):
            for x, w, y in calls:
                self.rb.matmul(x, w, out=y)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / reps
        return "w8a8 gemm_kernel + row quantiser (qkv, o, fc1, fc2 of one layer)", ops / (ms / 1e3) / 1e12, ms

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        """The reference CPU algorithm for one layer: the four W8A8 projections
        on 256 patch rows and the attention of 2 of 16 heads over one 2394-patch
        image, scaled to 27 layers x all rows / heads."""
        from burn_rocket_b200.siglip import SiglipConfig
        cfg = SiglipConfig()
        rng = np.random.default_rng(seed)
        rows, h, S, D = 256, cfg.hidden, cfg.patches, cfg.head_dim
        shapes = [(3 * h, h), (h, h), (cfg.inter, h), (h, cfg.inter)]
        ws = [orc.quantize_weight_per_channel((rng.standard_normal(sh) * 0.02).astype(np.float32)) for sh in shapes]
        xs = [rng.standard_normal((rows, sh[1])).astype(np.float32) for sh in shapes]
        q = rng.standard_normal((S, 2 * D)).astype(np.float32)
        kv = rng.standard_normal((S, 2 * D)).astype(np.float32)
        t0 = time.perf_counter()
        for _ in range(timed_repeats):
            for (codes, ws_), x in zip(ws, xs):
                orc.w8a8_matmul(x, codes, ws_)
        t_proj = (time.perf_counter() - t0) / timed_repeats / rows
        t0 = time.perf_counter()
        for _ in range(timed_repeats):
            orc.attention_cpu(q, kv, kv, 2, 2, D, 1 / math.sqrt(D), False)
        t_att = (time.perf_counter() - t0) / timed_repeats / S * (cfg.heads / 2)
        return 1.0 / ((t_proj + t_att) * cfg.layers), (
            "one layer: 4 W8A8 projections on 256 rows + attention of 2 of 16 heads over one image, x27 layers")


class MoeWorkload:
    """Config #5: Qwen3-30B-A3B-style MoE prefill, 4 sequences x 2048 tokens,
    48 layers, 128 experts top-8, causal. One GPU holds the whole model
    (~31 GB of Q8_0 weights)."""
    name = "moe"
    metric = "Qwen3-30B-A3B-style MoE prefill tok/s (config #5: 4 seq x 2048 tok, 48 layers, 128 experts top-8)"
    unit = "tok/s"
    BATCH, SEQ = 4, 2048
    LAYERS = None  # --layers: fewer decoder layers, for small ncu captures of the same kernels

    def __init__(self, dev, seed, world=1, rank=0):
        import torch
        from dataclasses import replace
        import burn_rocket_b200 as rb
        from burn_rocket_b200.moe import MoeConfig, MoeModel
        self.rb = rb
        self.cfg = MoeConfig() if self.LAYERS is None else replace(MoeConfig(), layers=self.LAYERS)
        if self.LAYERS is not None:
            self.metric = self.metric + f" [profiling case: {self.LAYERS} layers, not config #5]"
        self.world = world
        g = torch.Generator(device="cpu").manual_seed(seed)
        ids = torch.randint(0, self.cfg.vocab, (self.BATCH * self.SEQ,), generator=g, dtype=torch.int32)
        if world == 1:
            self.model = MoeModel(self.cfg, self.BATCH, self.SEQ, seed=0)
            mine = ids
        else:
            # expert parallelism: experts split over the ranks, tokens by sequence
            # (world <= 4) or by half sequence (world 8)
            import torch.distributed as dist
            from burn_rocket_b200.moe_ep import MoeEPModel, ep_plan
            pairs = ([dist.new_group([2 * i, 2 * i + 1]) for i in range(world // 2)]
                     if world > self.BATCH else None)
            # fixed-capacity all-to-alls: no host reads, the whole forward replays from a CUDA graph
            self.model = MoeEPModel(self.cfg, self.BATCH, self.SEQ, rank, world, seed=0, pair_groups=pairs)
            mine = torch.cat([ids[s * self.SEQ + r0: s * self.SEQ + r0 + n]
                              for s, r0, n in ep_plan(world, self.BATCH, self.SEQ)[rank]])
        self.model.ids_in.copy_(mine.to(dev))
        if world > 1:
            # exchange capacity from one exact forward over these inputs (outside any timing)
            self.model.calibrate_capacity()
        self.hids = mine.pin_memory()
        self.hout = torch.empty(self.model.T, self.cfg.hidden, dtype=torch.float16).pin_memory()
        self.units = self.model.T  # tokens per step on this rank
        self.flops = self.cfg.flops_per_token(self.SEQ) * self.units

    def step(self):
        self.model.forward_device()

    def e2e_step(self):
        if self.model.graph is None:  # the public host call replays the model's CUDA graph
            self.model.capture()
        self.model.prefill_host(self.hids, self.hout)
        return (self.hids.numel() * 4, self.hout.numel() * 2)

    def exchange_ms(self, barrier):
        """Expert parallelism: device time (max over ranks) of one step's
        all-to-alls alone — per layer the rows and expert ids out and the
        outputs back, on the model's own fixed-capacity buffers."""
        if self.world == 1:
            return None
        import torch
        import torch.distributed as dist
        from burn_rocket_b200.moe_ep import exchange
        m = self.model

        n = self.world * m.capacity

        def step():
            for _ in range(self.cfg.layers):
                exchange(m.recv_rows[:n], m.send_rows[:n], None, None, m.group)
                exchange(m.recv_meta[:n], m.send_meta[:n], None, None, m.group)
                exchange(m.y_back[:n], m.y_recv[:n], None, None, m.group)
        step()
        barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        reps = 3
        ev[0].record()
        for _ in range(reps):
            step()
        ev[1].record()
        barrier()
        t = torch.tensor([ev[0].elapsed_time(ev[1]) / reps], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def kernel_roofline(self):
        """Device time of one layer's grouped expert GEMMs (gate|up and down);
        None under expert parallelism (the whole step is reported)."""
        if self.world != 1:
            return None
        import torch
        import burn_rocket_b200._lib as L
        m, lay, lib = self.model, self.model.layers[0], L.load()
        cfg = self.cfg
        # routing of the current inputs for layer 0 is in the model's buffers after a forward
        ops = 2.0 * self.units * cfg.top_k * 3 * cfg.hidden * cfg.inter

        def run():
            lib.rb_matmul_grouped(lay["gu"].id, cfg.experts, m.xp.data_ptr(), m.max_rows, m.ws.data_ptr(), m.T,
                                  cfg.top_k, (m.actp if m.gated else m.gup).data_ptr(), L.DTYPE_F16, None)
            lib.rb_matmul_grouped(lay["down"].id, cfg.experts, m.actp.data_ptr(), m.max_rows, m.ws.data_ptr(), m.T,
                                  cfg.top_k, m.yp.data_ptr(), L.DTYPE_F16, None)
        for _ in range(2):
            run()
        reps = 5
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(reps):
            run()
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / reps
        return "grouped q8_0 gemm_pair_kernel (experts gate|up + down of one layer)", ops / (ms / 1e3) / 1e12, ms

    @staticmethod
    def cpu_sample(orc, seed, timed_repeats=1):
        """The reference CPU algorithm for the routed experts of one layer on a
        256-token sample (dequantise + f32 GEMMs of the 8 selected experts per
        token, grouped per expert), scaled to 48 layers; the dense part is
        timed like Qwen3's (q/k/v/o projections + attention over 2048 tokens)."""
        from burn_rocket_b200.moe import MoeConfig
        cfg = MoeConfig()
        rng = np.random.default_rng(seed)
        T, h, i = 256, cfg.hidden, cfg.inter
        per_expert = T * cfg.top_k // cfg.experts  # 16 rows per expert on average
        gate = orc.q8_0_quantize((rng.standard_normal((2 * i, h)) * 0.02).astype(np.float32))
        down = orc.q8_0_quantize((rng.standard_normal((h, i)) * 0.02).astype(np.float32))
        xe = rng.standard_normal((per_expert, h)).astype(np.float32)
        ae = rng.standard_normal((per_expert, i)).astype(np.float32)
        t0 = time.perf_counter()
        for _ in range(cfg.experts // 8):  # 16 of the 128 experts, scaled
            orc.q8_0_matmul_cpu(xe, *gate)
            orc.q8_0_matmul_cpu(ae, *down)
        t_exp = (time.perf_counter() - t0) * 8 / T
        shapes = [((cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim, h), (h, cfg.heads * cfg.head_dim)]
        ws = [orc.q8_0_quantize((rng.standard_normal(sh) * 0.02).astype(np.float32)) for sh in shapes]
        xs = [rng.standard_normal((T, sh[1])).astype(np.float32) for sh in shapes]
        q = rng.standard_normal((512, 2 * cfg.head_dim)).astype(np.float32)
        kv = rng.standard_normal((512, cfg.head_dim)).astype(np.float32)
        t0 = time.perf_counter()
        for (codes, scales), x in zip(ws, xs):
            orc.q8_0_matmul_cpu(x, codes, scales)
        t_dense = (time.perf_counter() - t0) / T
        t0 = time.perf_counter()
        orc.attention_cpu(q, kv, kv, 2, 1, cfg.head_dim, 1 / math.sqrt(cfg.head_dim), True)
        # 2 of 32 heads over 512 of 2048 tokens (causal work grows with S^2)
        t_att = (time.perf_counter() - t0) * 16 * 16 / 2048
        return 1.0 / ((t_exp + t_dense + t_att) * cfg.layers), (
            "one layer: 16 of 128 experts on 16 rows each, q|k|v + o on 256 tokens, 2 of 32 heads of causal "
            "attention over 512 tokens; scaled to 48 layers and 2048-token sequences")


WORKLOADS = {w.name: w for w in (AttnWorkload, Q8GemmWorkload, W8A8Workload, W8A8GroupWorkload, Qwen3Workload,
                                 SiglipWorkload, MoeWorkload)}
DP_WORKLOADS = ("qwen3", "siglip", "moe")


# ----------------------------------------------------------------------------- driver
def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return rank, world, local


def config_dict(name, world):
    """The `config` object of a workload's line; both arms print the same one."""
    return {"workload": {"attn": "configs[1] GQA attention", "q8gemm": "configs[0] Q8_0 GEMM",
                         "w8a8": "configs[3] W8A8 projections",
                         "w8a8g": "configs[3] projections, group-wise int8 g128",
                         "qwen3": "configs[2] Qwen3-Embedding-0.6B arch, 28 layers, 64x512 tokens",
                         "siglip": "configs[3] SigLIP-style W8A8 tower, 27 layers, 16x2394 patches",
                         "moe": "configs[4] Qwen3-30B-A3B-style MoE, 48 layers, 4x2048 tokens"}[name],
            "l2": L2_NOTE.get(name, "flushed between timed steps (256 MiB write)") if name not in SINGLE_OPS
                  else "inputs larger than L2: steps back to back over input/weight copies exceeding 2 x L2",
            "parallelism": (f"dp{world} over sequences" if name == "qwen3"
                            else f"dp{world} over images" if name == "siglip"
                            else ("single GPU, all 128 experts resident" if world == 1
                                  else f"ep{world} (experts {128 // world}/rank, NCCL all-to-all), "
                                       f"{'dp over sequences' if world <= 4 else 'half sequences'}")
                            if name == "moe"
                            else (f"replicas x{world}" if world > 1 else "single GPU"))}


DTYPES = {"attn": "f16", "q8gemm": "f16xq8_0->f32", "w8a8": "s8", "w8a8g": "s8 (group-wise, g128)", "qwen3": "f16xq8_0 (f32 residual)",
          "siglip": "s8 linears, f16 attention (f32 residual)", "moe": "f16xq8_0 (f32 residual, f32 router)"}
DEFAULT_STEPS = {"attn": 200, "q8gemm": 2000, "w8a8": 60, "w8a8g": 30, "qwen3": 20, "siglip": 5, "moe": 3}
# Single ops: steps run back to back, cycling over independent input sets
# (weights included) whose bytes together exceed twice the 126 MB L2, so no
# step finds its inputs in L2 and no flush or per-step event pair sits
# between them (w8a8 / w8a8g touch over 1 GB per step: one set).
SINGLE_OPS = ("q8gemm", "attn", "w8a8", "w8a8g")
L2_BYTES = 126e6
L2_NOTE = {}  # workload -> the `l2` note of its last single-op measurement


def footprint_bytes(wl):
    """Device bytes one step of a single-op workload touches: its CUDA
    tensors plus the resident weights it names in `weight_bytes`."""
    import torch
    tot = float(getattr(wl, "weight_bytes", 0))
    for v in vars(wl).values():
        for t in (v if isinstance(v, (list, tuple)) else [v]):
            if isinstance(t, torch.Tensor) and t.is_cuda:
                tot += t.numel() * t.element_size()
    return tot


def input_copies(wl):
    """Independent input sets so that their bytes exceed 2 x L2 (at most 32)."""
    return int(min(32, max(1, math.ceil(2 * L2_BYTES / max(footprint_bytes(wl), 1.0)))))


def l2_note(C, fp):
    if C == 1:
        return f"inputs larger than L2: {fp / 1e6:.0f} MB per step, steps back to back"
    return f"inputs larger than L2: steps back to back over {C} input/weight copies ({C * fp / 1e6:.0f} MB)"
# configs[0], [1] and [3]'s projections: measured beside the default (config #3) line at N = 1
SUB_WORKLOADS = ("q8gemm", "attn", "w8a8", "w8a8g")


def time_device(wl, steps, warmup, flush, stream, use_graph, barrier, local):
    """W untimed warm-ups, then exactly `steps` steps timed with CUDA events on
    the launching stream (an L2 flush between them, outside the events), with
    NVML clock sampling during the timed region. One step = the workload's
    C-ABI calls, captured once into a CUDA graph so host-side Python/ctypes
    overhead stays out of the device timing. Returns (ms summed over the
    steps, kernel launches in the timed region, graph used, clock summary)."""
    import torch
    import burn_rocket_b200 as rb
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize()
    rb.check_device_errors()
    graph = None
    rb.launch_count(reset=True)
    per_step = 0
    if use_graph and getattr(wl, "graphable", True):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            wl.step()
        per_step = rb.launch_count(reset=True)
        graph.replay()
        torch.cuda.synchronize()
        rb.check_device_errors()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    with ClockSampler(local) as clocks:
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            if graph is not None:
                graph.replay()
            else:
                wl.step()
            ends[i].record(stream)
        barrier()
    launches = per_step * steps if graph is not None else rb.launch_count()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    rb.check_device_errors()
    del graph
    return ms, launches, per_step > 0, clocks.summary()


def time_single(wls, steps, warmup, stream, use_graph, local):
    """Single-op timing: W untimed warm-up steps, then exactly `steps` steps
    back to back between one pair of CUDA events on the launching stream,
    step i running on input set i % len(wls). The `steps` steps are captured
    as one CUDA graph, replayed once behind a short device-side sleep so that
    the host's launch is off the device timeline. Returns (ms summed over the steps, kernel launches in the timed
    region, graph used, clock summary)."""
    import torch
    import burn_rocket_b200 as rb
    C = len(wls)
    for i in range(max(warmup, C)):
        wls[i % C].step()
    torch.cuda.synchronize()
    rb.check_device_errors()
    rb.launch_count(reset=True)
    graph = None
    if use_graph and all(getattr(w, "graphable", True) for w in wls):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            for i in range(steps):
                wls[i % C].step()
        per_replay = rb.launch_count(reset=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        torch.cuda._sleep(2_000_000)  # ~1 ms
        start.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(steps):
                wls[i % C].step()
        end.record(stream)
        torch.cuda.synchronize()
    graphed = graph is not None
    launches = per_replay if graphed else rb.launch_count()
    ms = start.elapsed_time(end)
    rb.check_device_errors()
    del graph
    return ms, launches, graphed, clocks.summary()


def time_e2e(wl, steps, barrier):
    """Seconds for `steps` end-to-end calls through the public host entry
    points (pinned host buffers, copies inside), and their bytes per step."""
    for _ in range(2):
        wl.e2e_step()
    barrier()
    t0 = time.perf_counter()
    h2d = d2h = 0
    for _ in range(steps):
        h2d, d2h = wl.e2e_step()
    return time.perf_counter() - t0, h2d, d2h


def roofline_of(wl, ms_per_step, peaks, peak_kind):
    """Roofline of the workload's dominant kernel: the model workloads time
    their dominant GEMMs alone (inside a long step they run at the sustained
    clock, so against the sustained peak); the single ops use the whole step
    against the burst peak."""
    kr = wl.kernel_roofline() if hasattr(wl, "kernel_roofline") else None
    int8 = wl.name in ("w8a8", "w8a8g", "siglip")
    if kr is not None:
        kname, achieved, kms = kr
        peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
        peak_src = f"{peak_kind} MEASURED_PEAKS bf16_tflops_sustained"
    else:
        kname = "whole step"
        achieved = wl.flops / (ms_per_step / 1e3) / 1e12
        peak = float(peaks["bf16_tflops"])
        peak_src = f"{peak_kind} MEASURED_PEAKS bf16_tflops (burst)"
    if int8:
        peak = 2.0 * peak  # dense int8 is twice the dense bf16 rate
        peak_src += " x2 for int8"
    return {"bound": "tensor", "kernel": kname, "achieved": round(achieved, 2), "peak": peak,
            "unit": "TOP/s" if int8 else "TFLOP/s", "frac": round(achieved / peak, 4),
            "traffic": profile_traffic(wl.name), "peak_source": peak_src}


def cpu_baseline_of(W, orc):
    v, sample = W.cpu_sample(orc, seed=1)
    return {"value": round(v, 5), "unit": W.unit, "cores": orc.num_threads(), "kind": "port", "sample": sample}


def measure_sub(name, dev, flush, stream, args, peaks, peak_kind):
    """One single-op sub-record (config #1 / #2 / #4 projections) at N = 1
    (its cpu_baseline is added after every GPU measurement of the run)."""
    import torch
    W = WORKLOADS[name]
    wl = W(dev, seed=0x5EED)
    C, fp = input_copies(wl), footprint_bytes(wl)
    wls = [wl] + [W(dev, seed=0x5EED + i) for i in range(1, C)]
    L2_NOTE[name] = l2_note(C, fp)
    steps = DEFAULT_STEPS[name]
    ms, launches, graphed, clocks = time_single(wls, steps, args.warmup, stream, not args.no_graph, dev.index)
    ms_per_step = ms / steps
    value = wl.flops / 1e12 / (ms_per_step / 1e3)
    e2e_steps = 10
    e2e_s, h2d, d2h = time_e2e(wl, e2e_steps, torch.cuda.synchronize)
    rec = {"workload": config_dict(name, 1)["workload"], "metric": W.metric, "value": round(value, 3),
           "unit": W.unit, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
           "dtype": DTYPES[name], "roofline": roofline_of(wl, ms_per_step, peaks, peak_kind),
           "e2e": {"value": round(wl.flops / 1e12 * e2e_steps / e2e_s, 3), "unit": W.unit,
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
           "gpu_launches": int(launches), "clocks": clocks, "l2": L2_NOTE[name],
           "timing": ("one CUDA graph over the steps' C-ABI calls, back to back" if graphed
                      else "eager launches, back to back")}
    if hasattr(wl, "beside"):
        rec.update(wl.beside(stream, float(peaks["bf16_tflops"])))
    del wl, wls
    torch.cuda.empty_cache()
    return rec


def measure_dp_sub(name, dev, flush, stream, args, peaks, peak_kind, world, rank, barrier, reduce_max):
    """A data-parallel model sub-record (config #4's tower over 16/N images per
    rank), timed like the main line: max over ranks, aggregate value."""
    import torch
    W = WORKLOADS[name]
    wl = W(dev, seed=0x5EED, world=world, rank=rank)
    steps = DEFAULT_STEPS[name]
    ms, launches, graphed, clocks = time_device(wl, steps, args.warmup, flush, stream, not args.no_graph,
                                                barrier, dev.index)
    ms_max = reduce_max(ms)
    value = wl.units * world * steps / (ms_max / 1e3)
    e2e_steps = 3
    e2e_s, h2d, d2h = time_e2e(wl, e2e_steps, barrier)
    e2e_value = wl.units * world * e2e_steps / reduce_max(e2e_s)
    rec = {"workload": config_dict(name, world)["workload"], "metric": W.metric, "value": round(value, 3),
           "unit": W.unit, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_max / steps, 4),
           "scaling": "strong", "parallelism": config_dict(name, world)["parallelism"], "dtype": DTYPES[name],
           "roofline": roofline_of(wl, ms_max / steps, peaks, peak_kind),
           "e2e": {"value": round(e2e_value, 3), "unit": W.unit, "h2d_bytes_per_step": int(h2d),
                   "d2h_bytes_per_step": int(d2h)},
           "gpu_launches": int(launches), "clocks": clocks,
           "timing": "CUDA-graph replay of the step's C-ABI calls" if graphed else "eager launches"}
    if hasattr(wl, "exchange_ms"):
        a2a = wl.exchange_ms(barrier)
        if a2a is not None:
            rec["alltoall"] = {"ms_per_step": round(a2a, 4), "share_of_step": round(a2a / (ms_max / steps), 4),
                               "what": "per layer: token rows + expert ids out, expert outputs back "
                                       f"(NCCL all_to_all_single, fixed capacity {wl.model.capacity} rows "
                                       f"per destination of the rank's {wl.model.S} routed slots, calibrated "
                                       "from an exact forward over the inputs), timed alone"}
    wl.model.graph = None  # release the graph (NCCL calls inside) before the process group
    del wl
    torch.cuda.empty_cache()
    return rec


def run_b200(args):
    import torch
    import torch.distributed as dist
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import burn_rocket_b200 as rb
    rb.init(local)
    rb.set_tile_policy(args.tile_policy)
    W = WORKLOADS[args.workload]
    wl = W(dev, seed=0x5EED, world=world, rank=rank) if W.name in DP_WORKLOADS else W(dev, seed=0x5EED + rank)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    if wl.name in SINGLE_OPS:
        barrier()
        C, fp = input_copies(wl), footprint_bytes(wl)
        L2_NOTE[wl.name] = l2_note(C, fp)
        wls = [wl] + [W(dev, seed=0x5EED + rank + 1000 * i) for i in range(1, C)]
        ms, launches, graphed, clocks = time_single(wls, args.steps, args.warmup, stream, not args.no_graph, local)
        barrier()
        del wls
    else:
        ms, launches, graphed, clocks = time_device(wl, args.steps, args.warmup, flush, stream, not args.no_graph,
                                                    barrier, local)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    # metric units per step per rank: TFLOP (TOP) for the op workloads, tokens for qwen3
    per_step = wl.units if hasattr(wl, "units") else wl.flops / 1e12
    value = per_step * world * args.steps / (ms_max / 1e3)

    # End-to-end through the host entry points (copies inside the timed region).
    e2e_steps = max(3, min(args.steps, 10))
    e2e_s, h2d, d2h = time_e2e(wl, e2e_steps, barrier)
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = per_step * world * e2e_steps / float(te.item())

    peaks, peak_kind = load_peaks()
    line = {
        "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong" if wl.name in DP_WORKLOADS else "weak", "vs_baseline": None,
        "dtype": DTYPES[wl.name],
        "data": "synthetic (seeded, BASELINE.json shapes)",
        "config": config_dict(wl.name, world),
        "roofline": roofline_of(wl, ms_per_step, peaks, peak_kind),
        "e2e": {"value": round(e2e_value, 3), "unit": wl.unit, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": int(launches),
        **({"l2": L2_NOTE[wl.name]} if wl.name in L2_NOTE else {}),
        "timing": ("one CUDA graph over the steps' C-ABI calls, back to back" if graphed and wl.name in SINGLE_OPS
                   else "CUDA-graph replay of the step's C-ABI calls" if graphed
                   else "eager launches (per-layer host-sized all-to-all)" if wl.name == "moe" and world > 1
                   else "eager launches"),
        "clocks": clocks,
    }
    if world > 1:
        dist.barrier()
    if args.workload == "qwen3" and not args.no_sub:
        del wl
        torch.cuda.empty_cache()

        def reduce_max(v):
            t = torch.tensor([v], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        # config #4's tower, data-parallel over images like the main line (every N)
        line["sub"] = {"siglip": measure_dp_sub("siglip", dev, flush, stream, args, peaks, peak_kind, world, rank,
                                                barrier, reduce_max)}
        if world > 1:
            # config #5's MoE, its experts spread over the N GPUs (expert parallelism)
            line["sub"]["moe_ep"] = measure_dp_sub("moe", dev, flush, stream, args, peaks, peak_kind, world, rank,
                                                   barrier, reduce_max)
        if world == 1:
            # the metric's single-op items, each timed alone on this GPU
            for name in SUB_WORKLOADS:
                line["sub"][name] = measure_sub(name, dev, flush, stream, args, peaks, peak_kind)
    # The host-core baselines run after every GPU measurement, so that their
    # OpenMP threads share no time with a timed region.
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        orc.use_all_host_cores()
        line["cpu_baseline"] = cpu_baseline_of(W, orc)
        for name, rec in line.get("sub", {}).items():
            if name in SUB_WORKLOADS:
                rec["cpu_baseline"] = cpu_baseline_of(WORKLOADS[name], orc)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 alone runs the host-core reference
    from oracle import oracle as orc
    # torchrun sets OMP_NUM_THREADS=1 in every rank: use all host cores anyway
    orc.use_all_host_cores()
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))

    def run(W, steps, warmup):
        for _ in range(warmup):
            W.cpu_sample(orc, seed=1)
        vals, sample = [], ""
        t0 = time.perf_counter()
        for _ in range(steps):
            v, sample = W.cpu_sample(orc, seed=1)
            vals.append(v)
        return statistics.median(vals), sample, (time.perf_counter() - t0) / steps

    W = WORKLOADS[args.workload]
    value, sample, s_per_step = run(W, args.steps, args.warmup)
    note = ("CPU restatement of the reference's --device cpu algorithm (oracle/, OpenMP on all host cores); "
            "the Rust reference cannot be built here (no cargo/rustc, no crate registry)")
    line = {
        "impl": "reference", "metric": W.metric, "value": round(value, 5), "unit": W.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(s_per_step * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if W.name in DP_WORKLOADS else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE.json shapes)",
        "config": config_dict(W.name, world),
        "cpu_baseline": {"value": round(value, 5), "unit": W.unit, "cores": orc.num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": W.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note,
    }
    if args.workload == "qwen3" and not args.no_sub:
        line["sub"] = {}
        for name in SUB_WORKLOADS:
            S = WORKLOADS[name]
            v, smp, sps = run(S, 3, 1)
            line["sub"][name] = {"workload": config_dict(name, 1)["workload"], "metric": S.metric,
                                 "value": round(v, 5), "unit": S.unit, "steps": 3, "warmup": 1,
                                 "ms_per_step": round(sps * 1e3, 3),
                                 "cpu_baseline": {"value": round(v, 5), "unit": S.unit, "cores": orc.num_threads(),
                                                  "kind": "port", "sample": smp}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: per workload, ~0.1-1 s)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="qwen3", choices=sorted(WORKLOADS),
                    help="default qwen3 (configs[2], the metric's model item) with sub-records for configs[0], "
                         "[1] and [3]'s projections at N = 1")
    ap.add_argument("--no-sub", action="store_true", help="qwen3: skip the single-op sub-records")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying a CUDA graph")
    ap.add_argument("--tile-policy", default="auto", choices=["auto", "single", "pair"],
                    help="GEMM tile policy (rb_set_tile_policy)")
    ap.add_argument("--layers", type=int, default=None,
                    help="moe: build only this many decoder layers (small ncu captures of the model's kernels; "
                         "the line is then not config #5)")
    ap.add_argument("--gemm-shape", default=None,
                    help="q8gemm / w8a8: one M,N,K GEMM with f16 activations/outputs (profiling the model's shapes)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.steps is None:
        args.steps = DEFAULT_STEPS.get(args.workload, 20)
    if args.gemm_shape:
        m, n, k = (int(v) for v in args.gemm_shape.split(","))
        if args.workload == "w8a8":
            W8A8Workload.M, W8A8Workload.SHAPES = m, [(n, k)]
            W8A8Workload.X_DTYPE = "f16"
        else:
            Q8GemmWorkload.M, Q8GemmWorkload.N, Q8GemmWorkload.K = m, n, k
            Q8GemmWorkload.X_DTYPE = "f16"
    if args.layers is not None:
        if args.workload != "moe" or args.layers < 1:
            ap.error("--layers applies to --workload moe, with at least one layer")
        MoeWorkload.LAYERS = args.layers
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
