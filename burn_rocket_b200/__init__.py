"""burn_rocket_b200 — B200 (sm_100a) drop-in for the ops burn-rocket offloads.

The operator surface mirrors burn-rocket's helpers over its `RocketOps`
backend extension (crates/burn-rocket/src/ext.rs:1866-2137, re-exported at
lib.rs:34-42): `init`, `pack`/`pack2`/`pack3` (Q8_0 resident weights),
`pack_qat` (per-channel W8A8), `matmul`, and the `attention*` family, with
the same argument meaning. Failures raise `OpFailure` carrying the reference's
`Error{op, rc}` and the call's shape (lib.rs:116-167), as the reference's ops
panic with an `OpFailure` payload (ext.rs:344-352).

All compute runs in librocket_b200.so (hand-written sm_100a kernels behind a
C ABI, include/rocket_b200.h). torch is used only to hold device memory and
streams; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import (DTYPE_BF16, DTYPE_F16, DTYPE_F32, MASK_CAUSAL, MASK_CAUSAL_BLOCK,
                   MASK_CAUSAL_WINDOW, MASK_NONE, MASK_NONE_BLOCK, MASK_WINDOW,
                   MASK_WINDOW_BLOCK, WEIGHT_Q8_0, WEIGHT_W8A8)

__all__ = [
    "Error", "OpFailure", "WeightId", "init", "pack", "pack2", "pack3", "pack_q8_0", "pack2_q8_0", "pack3_q8_0",
    "pack_q8_0_blocks", "pack_w8a8_float",
    "pack_i8", "quantize_row_groups",
    "pack_qat", "matmul", "matmul_host", "attention", "attention_window",
    "attention_causal_window", "attention_window_block", "attention_causal_block",
    "attention_raw", "q8_0_dequant", "quantize_rows_i8", "matmul_i8_acc", "check_device_errors",
    "mem_stats", "launch_count",
]


@dataclass(frozen=True)
class Error:
    """A failed operation: the op name and the negative status code (lib.rs:116-146)."""
    op: str
    rc: int

    def is_fallback(self) -> bool:
        return self.rc == _lib.RB_E_TILING

    def __str__(self) -> str:
        return f"{self.op} failed: {_lib.RC_NAMES.get(self.rc, 'unknown error')} (rc={self.rc})"


class OpFailure(RuntimeError):
    """Raised by a failed op: the `Error` plus the shape of the call (lib.rs:158-167)."""

    def __init__(self, error: Error, m: int = 0, k: int = 0, n: int = 0, detail: str = ""):
        self.error, self.m, self.k, self.n, self.detail = error, m, k, n, detail
        super().__init__(f"{error} m={m} k={k} n={n}: {detail}")


@dataclass(frozen=True)
class WeightId:
    """Handle of a resident weight (ext.rs:39-50). Valid for the process lifetime."""
    id: int


def _check(rc: int, op: str, m: int = 0, k: int = 0, n: int = 0) -> int:
    if rc < 0:
        raise OpFailure(Error(op, int(rc)), m, k, n, _lib.last_error())
    return rc


_DT = {}


def _dtype_code(t) -> int:
    import torch
    if not _DT:
        _DT.update({torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16})
    try:
        return _DT[t.dtype]
    except KeyError:
        raise OpFailure(Error("dtype", _lib.RB_E_SHAPE), detail=f"unsupported dtype {t.dtype}")


def _stream_ptr(stream) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _dev_ptr(t) -> int:
    if not t.is_cuda:
        raise OpFailure(Error("device", _lib.RB_E_SHAPE), detail="expected a CUDA tensor")
    if not t.is_contiguous():
        raise OpFailure(Error("layout", _lib.RB_E_SHAPE), detail="expected a contiguous tensor")
    return int(t.data_ptr())


# ----------------------------------------------------------------------------- init / pack
def init(device: int = 0) -> None:
    """Create the engine on CUDA device `device` (burn_rocket::init, ext.rs:561-580)."""
    _check(_lib.load().rb_init(int(device)), "rb_init")


def _as_f32_host(w) -> np.ndarray:
    if hasattr(w, "detach"):
        w = w.detach().float().cpu().numpy()
    return np.ascontiguousarray(np.asarray(w, dtype=np.float32))


def _pack_parts_q8_0(parts: Sequence) -> WeightId:
    arrs = [_as_f32_host(p) for p in parts]
    k = arrs[0].shape[1]
    for a in arrs:
        if a.ndim != 2 or a.shape[1] != k:
            raise OpFailure(Error("rocket_pack", _lib.RB_E_SHAPE), detail="all parts must be [N_i, K] with a shared K")
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    ns = (C.c_int64 * len(arrs))(*[a.shape[0] for a in arrs])
    wid = _lib.load().rb_pack_f32_q8_0(ptrs, ns, len(arrs), k)
    _check(wid, "rocket_pack", 0, k, sum(a.shape[0] for a in arrs))
    return WeightId(int(wid))


def _pack_parts_f16(parts: Sequence) -> WeightId:
    """Host parts (numpy / CPU torch tensors of f32, f16 or bf16) -> one fp16-resident weight."""
    import torch
    ts = []
    for p in parts:
        t = p.detach() if hasattr(p, "detach") else torch.from_numpy(np.ascontiguousarray(p))
        t = t.cpu()
        if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            t = t.float()
        ts.append(t.contiguous())
    dt = ts[0].dtype
    ts = [t.to(dt) for t in ts]
    k = ts[0].shape[1]
    for t in ts:
        if t.dim() != 2 or t.shape[1] != k:
            raise OpFailure(Error("rocket_pack", _lib.RB_E_SHAPE), detail="all parts must be [N_i, K] with a shared K")
    ptrs = (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    ns = (C.c_int64 * len(ts))(*[t.shape[0] for t in ts])
    wid = _lib.load().rb_pack_f16(ptrs, ns, len(ts), k, _dtype_code(ts[0]))
    _check(wid, "rocket_pack", 0, k, sum(t.shape[0] for t in ts))
    return WeightId(int(wid))


def pack(w) -> WeightId:
    """Pack an [N, K] float weight as a resident fp16 weight (rocket_pack, ext.rs:59, 829-850)."""
    return _pack_parts_f16([w])


def pack2(a, b) -> WeightId:
    """Pack two fp16 weights sharing one input, concatenated along N (ext.rs:61)."""
    return _pack_parts_f16([a, b])


def pack3(a, b, c) -> WeightId:
    """Pack three fp16 weights sharing one input, concatenated along N (ext.rs:63)."""
    return _pack_parts_f16([a, b, c])


def pack_q8_0(w) -> WeightId:
    """Pack an [N, K] float weight as a resident Q8_0 weight (the GGUF Q8_0 route:
    device encoder of q8_bench.rs:199-219; dequantised inside the GEMM)."""
    return _pack_parts_q8_0([w])


def set_weight_activation(w: WeightId, act: str) -> None:
    """Fuse an element-wise activation into later matmuls on weight `w`
    ("gelu_tanh", host.rs:15-18, or "none"); the output must then be f16."""
    names = {"none": 0, "gelu_tanh": 1}
    if act not in names:
        raise ValueError(f"activation must be one of {list(names)}")
    _check(_lib.load().rb_set_weight_activation(w.id, names[act]), "rb_set_weight_activation")


def pack_gated_q8_0(gate, up) -> WeightId:
    """SwiGLU gate|up as one Q8_0 weight whose matmul returns the fused
    f16 silu(x gate^T) * (x up^T) ([M, n_inter]; host.rs:31-38), i.e. the
    pack2 gate|up matmul and silu_mul of a SwiGLU MLP in one kernel. gate and
    up are [n_inter, K] float tensors (n_inter a multiple of 64); stacked
    per-expert blocks give a gated grouped weight."""
    import torch
    lib = _lib.load()
    g = gate.detach().to("cuda", torch.float32).contiguous()
    u = up.detach().to("cuda", torch.float32).contiguous()
    if g.shape != u.shape or g.dim() != 2:
        raise OpFailure(Error("rocket_pack2", _lib.RB_E_SHAPE), 0, 0, 0, "gate and up must be equal [n, K]")
    wid = lib.rb_pack_f32_q8_0_gated_device(g.data_ptr(), u.data_ptr(), g.shape[0], g.shape[1])
    _check(wid, "rocket_pack2", 0, g.shape[1], 2 * g.shape[0])
    return WeightId(int(wid))


def pack2_q8_0(a, b) -> WeightId:
    return _pack_parts_q8_0([a, b])


def pack3_q8_0(a, b, c) -> WeightId:
    return _pack_parts_q8_0([a, b, c])


def pack_q8_0_blocks(blocks: np.ndarray, n: int, k: int) -> WeightId:
    """Pack GGUF Q8_0 blocks (34 B each, util/gguf.rs:197-215) of an [n, k] weight."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    if blocks.size != n * (k // 32) * 34:
        raise OpFailure(Error("rb_pack_q8_0", _lib.RB_E_SHAPE), 0, k, n, "block buffer size mismatch")
    wid = _lib.load().rb_pack_q8_0(blocks.ctypes.data, n, k)
    _check(wid, "rb_pack_q8_0", 0, k, n)
    return WeightId(int(wid))


def pack_qat(codes, w_scale, n: int, k: int, in_scale: float = 0.0, out_scale: float = 0.0) -> WeightId:
    """Per-output-channel int8 weight (burn_rocket::pack_qat, ext.rs:1382-1425)."""
    codes = np.ascontiguousarray(np.asarray(codes, dtype=np.int8))
    w_scale = np.ascontiguousarray(np.asarray(w_scale, dtype=np.float32))
    if codes.size != n * k:
        raise OpFailure(Error("rocket_pack_qat", _lib.RB_E_SHAPE), 0, k, n, "QAT codes must be [N, K]")
    if w_scale.size != n:
        raise OpFailure(Error("rocket_pack_qat", _lib.RB_E_SHAPE), 0, k, n, "one weight scale per output channel")
    wid = _lib.load().rb_pack_w8a8(codes.ctypes.data, w_scale.ctypes.data, n, k, float(in_scale), float(out_scale))
    _check(wid, "rocket_pack_qat", 0, k, n)
    return WeightId(int(wid))


def pack_i8(w, group: int) -> WeightId:
    """Pack an [N, K] float weight as a group-wise int8 weight (rocket_pack_i8,
    ext.rs:939-1029); rb_matmul then quantises the activations per group too."""
    a = _as_f32_host(w)
    if a.ndim != 2:
        raise OpFailure(Error("rocket_pack_i8", _lib.RB_E_SHAPE), detail="weight must be [N, K]")
    n, k = a.shape
    wid = _lib.load().rb_pack_i8(a.ctypes.data, n, k, int(group))
    _check(wid, "rocket_pack_i8", 0, k, n)
    return WeightId(int(wid))


def quantize_row_groups(x, group: int):
    """Device group-wise row quantiser (host.rs:77-90): (codes int8 [M, K], scales f32 [M, K/group])."""
    import torch
    x = x.contiguous()
    m, k = x.reshape(-1, x.shape[-1]).shape
    codes = torch.empty(m, k, dtype=torch.int8, device=x.device)
    scales = torch.empty(m, k // group, dtype=torch.float32, device=x.device)
    _check(_lib.load().rb_quantize_row_groups(_dev_ptr(x), _dtype_code(x), m, k, int(group), _dev_ptr(codes),
                                              _dev_ptr(scales), None), "quantize_row_groups")
    return codes, scales


def pack_w8a8_float(w, in_scale: float = 0.0, out_scale: float = 0.0) -> WeightId:
    """Quantise a float [N, K] CUDA weight to per-output-channel int8 on the
    device (rb_pack_f32_w8a8_device) and pack it like pack_qat."""
    import torch
    if not (isinstance(w, torch.Tensor) and w.is_cuda and w.dim() == 2):
        raise OpFailure(Error("rocket_pack_qat", _lib.RB_E_SHAPE), detail="weight must be a 2-D CUDA tensor")
    w = w.detach().float().contiguous()
    n, k = w.shape
    wid = _lib.load().rb_pack_f32_w8a8_device(C.c_void_p(w.data_ptr()), n, k, float(in_scale), float(out_scale))
    _check(wid, "rocket_pack_qat", 0, k, n)
    return WeightId(int(wid))


def weight_info(w: WeightId):
    kind, n, k = C.c_int(), C.c_int64(), C.c_int64()
    _check(_lib.load().rb_weight_info(w.id, C.byref(kind), C.byref(n), C.byref(k)), "rb_weight_info")
    return kind.value, n.value, k.value


# ----------------------------------------------------------------------------- matmul
def matmul(x, w: WeightId, out=None, out_dtype=None, stream=None):
    """`x[.., M, K] @ W[N, K]^T -> [.., M, N]` with a resident weight (ext.rs:1899-1905).

    x is a CUDA tensor (f32/f16/bf16); the output dtype defaults to x's, as in
    the reference (ext.rs:1038-1052)."""
    import torch
    _, n, k = weight_info(w)
    if x.shape[-1] != k:
        raise OpFailure(Error("rocket_matmul", _lib.RB_E_SHAPE), 0, x.shape[-1], n, f"activation K mismatch (weight K={k})")
    m = int(np.prod(x.shape[:-1])) if x.dim() > 1 else 1
    x = x.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=out_dtype or x.dtype, device=x.device)
    rc = _lib.load().rb_matmul(w.id, _dev_ptr(x), _dtype_code(x), m, k, _dev_ptr(out), _dtype_code(out),
                               _stream_ptr(stream))
    _check(rc, "rocket_matmul", m, k, n)
    return out


def matmul_host(x: np.ndarray, w: WeightId, out_dtype=np.float32) -> np.ndarray:
    """matmul on HOST numpy arrays; the copies happen inside the C-ABI call."""
    _, n, k = weight_info(w)
    x = np.ascontiguousarray(x)
    dt = {np.dtype(np.float32): DTYPE_F32, np.dtype(np.float16): DTYPE_F16}[x.dtype]
    m = x.size // k
    y = np.empty((*x.shape[:-1], n), dtype=out_dtype)
    ydt = {np.dtype(np.float32): DTYPE_F32, np.dtype(np.float16): DTYPE_F16}[y.dtype]
    _check(_lib.load().rb_matmul_host(w.id, x.ctypes.data, dt, m, k, y.ctypes.data, ydt), "rocket_matmul", m, k, n)
    return y


# ----------------------------------------------------------------------------- attention
def attention_raw(q, k, v, n_head: int, n_kv_heads: int, head_dim: int, scale: float,
                  softcap: Optional[float], mask_mode: int, window: int = -1, q_start: int = 0,
                  kv_start: int = 0, out=None, stream=None):
    """Masked GQA attention over [.., S, H*D] CUDA tensors (attention_impl, ext.rs:1669-1858)."""
    import torch
    n_q = q.shape[-2]
    n_kv = k.shape[-2]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if q.shape[-1] != n_head * head_dim:
        raise OpFailure(Error("rocket_attention", _lib.RB_E_SHAPE), n_q, n_kv, head_dim, "q width must be n_head * head_dim")
    if k.shape[-1] != n_kv_heads * head_dim or v.shape != k.shape:
        raise OpFailure(Error("rocket_attention", _lib.RB_E_SHAPE), n_q, n_kv, head_dim, "k/v must be [1, S, KV*D]")
    if out is None:
        out = torch.empty_like(q)
    rc = _lib.load().rb_attention(_dev_ptr(q), _dev_ptr(k), _dev_ptr(v), _dev_ptr(out), _dtype_code(q), n_q, n_kv,
                                  n_head, n_kv_heads, head_dim, float(scale), float(softcap or 0.0), mask_mode,
                                  int(window), int(q_start), int(kv_start), _stream_ptr(stream))
    _check(rc, "rocket_flash_attn", n_q, n_kv, head_dim)
    return out


def attention(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap=None, is_causal=False, **kw):
    """rocket_attention (ext.rs:87-98): causal or full bidirectional."""
    return attention_raw(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap,
                         MASK_CAUSAL if is_causal else MASK_NONE, **kw)


def attention_window(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap=None, window=-1, **kw):
    """rocket_attention_window (ext.rs:99-112): |t - j| <= window, window < 0 = no mask."""
    return attention_raw(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap, MASK_WINDOW, window, **kw)


def attention_causal_window(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap=None, window=-1, **kw):
    """rocket_attention_causal_window (ext.rs:113-126): t - window < j <= t."""
    return attention_raw(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap, MASK_CAUSAL_WINDOW, window, **kw)


def attention_window_block(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap=None, window=-1,
                           q_start=0, kv_start=0, **kw):
    """rocket_attention_window_block (ext.rs:127-144)."""
    return attention_raw(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap, MASK_WINDOW_BLOCK, window,
                         q_start, kv_start, **kw)


def attention_causal_block(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap=None, window=-1,
                           q_start=0, kv_start=0, **kw):
    """rocket_attention_causal_block (ext.rs:145-163)."""
    return attention_raw(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap, MASK_CAUSAL_BLOCK, window,
                         q_start, kv_start, **kw)


# ----------------------------------------------------------------------------- codec surfaces
def q8_0_dequant(w: WeightId, out_dtype="f32", stream=None):
    import torch
    _, n, k = weight_info(w)
    dt = torch.float32 if out_dtype == "f32" else torch.float16
    out = torch.empty(n, k, dtype=dt, device="cuda")
    _check(_lib.load().rb_q8_0_dequant(w.id, _dev_ptr(out), _dtype_code(out), _stream_ptr(stream)), "rb_q8_0_dequant")
    return out


def quantize_rows_i8(x, stream=None):
    import torch
    m, k = x.shape
    codes = torch.empty(m, k, dtype=torch.int8, device=x.device)
    scales = torch.empty(m, dtype=torch.float32, device=x.device)
    _check(_lib.load().rb_quantize_rows_i8(_dev_ptr(x), _dtype_code(x), m, k, _dev_ptr(codes), _dev_ptr(scales),
                                           _stream_ptr(stream)), "rb_quantize_rows_i8", m, k)
    return codes, scales


def matmul_i8_acc(codes, w: WeightId, stream=None):
    import torch
    _, n, k = weight_info(w)
    m = codes.shape[0]
    acc = torch.empty(m, n, dtype=torch.int32, device=codes.device)
    _check(_lib.load().rb_matmul_i8_acc(w.id, _dev_ptr(codes), m, _dev_ptr(acc), _stream_ptr(stream)),
           "rb_matmul_i8_acc", m, k, n)
    return acc


def check_device_errors() -> None:
    _check(_lib.load().rb_check_device_errors(), "rb_check_device_errors")


def mem_stats():
    wb, sb, nw = C.c_int64(), C.c_int64(), C.c_int64()
    _check(_lib.load().rb_mem_stats(C.byref(wb), C.byref(sb), C.byref(nw)), "rb_mem_stats")
    return {"weights_bytes": wb.value, "scratch_bytes": sb.value, "num_weights": nw.value}


def set_tile_policy(policy: str) -> str:
    """GEMM tile policy for later matmuls: "auto", "single" (single-CTA tiles
    only) or "pair" (prefer 256-row CTA-pair tiles). Returns the previous one."""
    names = ["auto", "single", "pair"]
    if policy not in names:
        raise ValueError(f"tile policy must be one of {names}")
    old = _lib.load().rb_set_tile_policy(names.index(policy))
    _check(old, "rb_set_tile_policy")
    return names[old]


def set_attention_split(policy: str) -> str:
    """Attention work split for later calls: "auto", "never" (one CTA per
    query-slot pair and KV head) or "always" (one CTA per SM over equal shares
    of the key tiles). Returns the previous one."""
    names = ["auto", "never", "always"]
    if policy not in names:
        raise ValueError(f"attention split policy must be one of {names}")
    old = _lib.load().rb_set_attention_split(names.index(policy))
    _check(old, "rb_set_attention_split")
    return names[old]


def launch_count(reset: bool = False) -> int:
    return int(_lib.load().rb_launch_count(1 if reset else 0))
