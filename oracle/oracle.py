"""numpy front end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY. The parity tests, `__graft_entry__.smoke()` and
bench.py's CPU-baseline / reference arm import this module as the checker;
the product (burn_rocket_b200, librocket_b200.so) never does. Each function
restates a reference routine; the C source cites the file:line it follows.
Parity is pinned by the reference's golden vectors (tests/test_oracle_golden.py).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None

_p = C.c_void_p
_i64 = C.c_int64
_f = C.c_float
_i = C.c_int


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sig = {
            "orc_f32_to_f16": (C.c_uint16, [_f]),
            "orc_f16_to_f32": (_f, [C.c_uint16]),
            "orc_f64_to_f16": (C.c_uint16, [C.c_double]),
            "orc_f32_to_f16_array": (None, [_p, _p, _i64]),
            "orc_f16_to_f32_array": (None, [_p, _p, _i64]),
            "orc_q8_0_quantize": (None, [_p, _i64, _i64, _p, _p]),
            "orc_q8_0_to_blocks": (None, [_p, _p, _i64, _i64, _p]),
            "orc_q8_0_dequant_blocks": (None, [_p, _i64, _p]),
            "orc_q8_0_dequant": (None, [_p, _p, _i64, _i64, _p]),
            "orc_gemm_f64acc": (None, [_p, _p, _i64, _i64, _i64, _p]),
            "orc_q8_0_matmul_cpu": (None, [_p, _p, _p, _i64, _i64, _i64, _p, _p]),
            "orc_static_code": (C.c_int8, [_f, _f]),
            "orc_quantize_rows_i8": (None, [_p, _i64, _i64, _f, _p, _p]),
            "orc_gemm_i8": (_i, [_p, _p, _i64, _i64, _i64, _p]),
            "orc_w8a8_epilogue": (None, [_p, _p, _p, _i64, _i64, _f, _p]),
            "orc_quantize_weight_per_channel": (None, [_p, _i64, _i64, _p, _p]),
            "orc_quantize_row_groups": (None, [_p, _i64, _i64, _p, _p]),
            "orc_mask_visible": (_i, [_i, _i64, _i64, _i64, _i64, _i64]),
            "orc_fa_score": (_f, [_f, _f, _f, _f]),
            "orc_flash_attn_ref": (None, [_p, _p, _p, _i64, _i64, _i, _i, _i, _f, _f, _i, _i64, _i64, _i64, _p]),
            "orc_attention_cpu": (None, [_p, _p, _p, _i64, _i64, _i, _i, _i, _f, _i, _p]),
            "orc_num_threads": (_i, []),
            "orc_set_num_threads": (None, [_i]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- f16
def f32_to_f16_bits(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16_array(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f16_bits_to_f32(h) -> np.ndarray:
    h = _c(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_f16_to_f32_array(h.ctypes.data, out.ctypes.data, h.size)
    return out


def f64_to_f16_bits(v: float) -> int:
    return int(lib().orc_f64_to_f16(float(v)))


# ---------------------------------------------------------------- Q8_0
def q8_0_quantize(w):
    """(codes int8 [n,k], scale bits uint16 [n,k/32]) — q8_bench.rs:199-219."""
    w = _c(w, np.float32)
    n, k = w.shape
    codes = np.empty((n, k), np.int8)
    scales = np.empty((n, k // 32), np.uint16)
    lib().orc_q8_0_quantize(w.ctypes.data, n, k, codes.ctypes.data, scales.ctypes.data)
    return codes, scales


def q8_0_to_blocks(codes, scales) -> np.ndarray:
    codes = _c(codes, np.int8)
    scales = _c(scales, np.uint16)
    n, k = codes.shape
    out = np.empty(n * (k // 32) * 34, np.uint8)
    lib().orc_q8_0_to_blocks(codes.ctypes.data, scales.ctypes.data, n, k, out.ctypes.data)
    return out


def q8_0_dequant_blocks(blocks) -> np.ndarray:
    blocks = _c(blocks, np.uint8)
    nb = blocks.size // 34
    out = np.empty(nb * 32, np.float32)
    lib().orc_q8_0_dequant_blocks(blocks.ctypes.data, nb, out.ctypes.data)
    return out


def q8_0_dequant(codes, scales) -> np.ndarray:
    codes = _c(codes, np.int8)
    scales = _c(scales, np.uint16)
    n, k = codes.shape
    out = np.empty((n, k), np.float32)
    lib().orc_q8_0_dequant(codes.ctypes.data, scales.ctypes.data, n, k, out.ctypes.data)
    return out


def gemm_f64acc(a, w) -> np.ndarray:
    a = _c(a, np.float32)
    w = _c(w, np.float32)
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), np.float32)
    lib().orc_gemm_f64acc(a.ctypes.data, w.ctypes.data, m, n, k, out.ctypes.data)
    return out


def q8_0_matmul_cpu(a, codes, scales, wdeq_scratch=None) -> np.ndarray:
    """The reference's --device cpu Q8 algorithm: dequantise + f32 GEMM (timed baseline)."""
    a = _c(a, np.float32)
    codes = _c(codes, np.int8)
    scales = _c(scales, np.uint16)
    m, k = a.shape
    n = codes.shape[0]
    if wdeq_scratch is None:
        wdeq_scratch = np.empty((n, k), np.float32)
    out = np.empty((m, n), np.float32)
    lib().orc_q8_0_matmul_cpu(a.ctypes.data, codes.ctypes.data, scales.ctypes.data, m, n, k,
                              wdeq_scratch.ctypes.data, out.ctypes.data)
    return out


# ---------------------------------------------------------------- W8A8
def static_code(v: float, inv: float) -> int:
    return int(lib().orc_static_code(float(v), float(inv)))


def quantize_rows_i8(x, in_scale: float = 0.0):
    x = _c(x, np.float32)
    m, k = x.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().orc_quantize_rows_i8(x.ctypes.data, m, k, float(in_scale), q.ctypes.data, s.ctypes.data)
    return q, s


def gemm_i8(q, w) -> np.ndarray:
    q = _c(q, np.int8)
    w = _c(w, np.int8)
    m, k = q.shape
    n = w.shape[0]
    acc = np.empty((m, n), np.int32)
    rc = lib().orc_gemm_i8(q.ctypes.data, w.ctypes.data, m, n, k, acc.ctypes.data)
    if rc != 0:
        raise OverflowError("int8 accumulator left int32")
    return acc


def w8a8_epilogue(acc, row_scale, w_scale, out_scale: float = 0.0) -> np.ndarray:
    acc = _c(acc, np.int32)
    row_scale = _c(row_scale, np.float32)
    w_scale = _c(w_scale, np.float32)
    m, n = acc.shape
    y = np.empty((m, n), np.float32)
    lib().orc_w8a8_epilogue(acc.ctypes.data, row_scale.ctypes.data, w_scale.ctypes.data, m, n,
                            float(out_scale), y.ctypes.data)
    return y


def w8a8_matmul(x, codes, w_scale, in_scale: float = 0.0, out_scale: float = 0.0) -> np.ndarray:
    """matmul_qat end to end (ext.rs:1245-1373)."""
    q, rs = quantize_rows_i8(x, in_scale)
    return w8a8_epilogue(gemm_i8(q, codes), rs, w_scale, out_scale)


def quantize_weight_per_channel(w):
    w = _c(w, np.float32)
    n, k = w.shape
    codes = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    lib().orc_quantize_weight_per_channel(w.ctypes.data, n, k, codes.ctypes.data, s.ctypes.data)
    return codes, s


def quantize_row_groups(x, group: int):
    x = _c(x, np.float32)
    k = x.size
    q = np.empty(k, np.int8)
    s = np.empty(k // group, np.float32)
    lib().orc_quantize_row_groups(x.ctypes.data, k, group, q.ctypes.data, s.ctypes.data)
    return q, s


def matmul_gw(aq, a_s, bq, b_s, group: int) -> np.ndarray:
    """Group-wise int8 matmul (matmul_gw, crates/rocket-npu/src/matmul/int8.rs:641-672;
    promotion order of layout.rs:504-529): acc = 0; for g in order:
    acc += f32(a_s[m,g] * b_s[n,g]) * f32(exact int32 partial of group g), all f32."""
    aq, bq = np.asarray(aq, np.int8), np.asarray(bq, np.int8)
    m, k = aq.shape
    n = bq.shape[0]
    ng = k // group
    acc = np.zeros((m, n), np.float32)
    for g in range(ng):
        part = gemm_i8(aq[:, g * group:(g + 1) * group], bq[:, g * group:(g + 1) * group])
        scale = (np.asarray(a_s, np.float32)[:, g:g + 1] * np.asarray(b_s, np.float32)[None, :, g]).astype(np.float32)
        acc = (acc + (scale * part.astype(np.float32)).astype(np.float32)).astype(np.float32)
    return acc


def quantize_rows_groups(x, group: int):
    """quantize_row_groups over every row of x [m, k] -> (codes [m, k], scales [m, k/group])."""
    x = np.asarray(x, np.float32)
    m, k = x.shape
    q = np.empty((m, k), np.int8)
    s = np.empty((m, k // group), np.float32)
    for r in range(m):
        q[r], s[r] = quantize_row_groups(x[r], group)
    return q, s


# ---------------------------------------------------------------- attention
MASK_NONE, MASK_NONE_BLOCK, MASK_CAUSAL, MASK_WINDOW = 0, 1, 2, 3
MASK_CAUSAL_WINDOW, MASK_WINDOW_BLOCK, MASK_CAUSAL_BLOCK = 4, 5, 6


def mask_visible(mode, window, q0, k0, i, j) -> bool:
    return bool(lib().orc_mask_visible(mode, window, q0, k0, i, j))


def mask_matrix(mode, n_q, n_kv, window=-1, q0=0, k0=0) -> np.ndarray:
    return np.array([[mask_visible(mode, window, q0, k0, i, j) for j in range(n_kv)] for i in range(n_q)])


def fa_score(qk, scale, softcap, mask) -> float:
    return float(lib().orc_fa_score(float(qk), float(scale), float(softcap), float(mask)))


def flash_attn_ref(q16, k16, v16, n_head, n_kv_heads, head_dim, scale, softcap=0.0, mode=MASK_NONE,
                   window=-1, q0=0, k0=0) -> np.ndarray:
    """flash_attn_ref (attn/oneshot.rs:130-185) on token-major f16 bits; returns f16 bits."""
    q16 = _c(q16, np.uint16)
    k16 = _c(k16, np.uint16)
    v16 = _c(v16, np.uint16)
    n_q = q16.size // (n_head * head_dim)
    n_kv = k16.size // (n_kv_heads * head_dim)
    out = np.empty((n_q, n_head * head_dim), np.uint16)
    lib().orc_flash_attn_ref(q16.ctypes.data, k16.ctypes.data, v16.ctypes.data, n_q, n_kv, n_head,
                             n_kv_heads, head_dim, float(scale), float(softcap), mode, window, q0, k0,
                             out.ctypes.data)
    return out


def attention_cpu(q, k, v, n_head, n_kv_heads, head_dim, scale, causal) -> np.ndarray:
    """Tiled f32 online-softmax attention over all threads (timed CPU baseline)."""
    q = _c(q, np.float32)
    k = _c(k, np.float32)
    v = _c(v, np.float32)
    n_q = q.size // (n_head * head_dim)
    n_kv = k.size // (n_kv_heads * head_dim)
    out = np.empty((n_q, n_head * head_dim), np.float32)
    lib().orc_attention_cpu(q.ctypes.data, k.ctypes.data, v.ctypes.data, n_q, n_kv, n_head, n_kv_heads,
                            head_dim, float(scale), 1 if causal else 0, out.ctypes.data)
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())


def host_cores() -> int:
    """Cores this process may run on (what `nproc` reports)."""
    import os
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def use_all_host_cores() -> int:
    """Run later oracle calls on every host core, whatever OMP_NUM_THREADS says;
    returns the thread count now in effect."""
    lib().orc_set_num_threads(host_cores())
    return num_threads()
