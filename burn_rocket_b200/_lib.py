"""ctypes binding of librocket_b200.so (include/rocket_b200.h).

The shared library is the product; this module only declares its C
signatures. Loading fails loudly when the library is missing: there is no
CPU fallback anywhere in the package.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librocket_b200.so"

# Status codes (lib.rs:116-146, rocket-npu error.rs:28-55).
RB_OK = 0
RB_E_SHAPE = -1
RB_E_TILING = -2
RB_E_NOMEM = -3
RB_E_DEVICE = -4
RB_E_UNSUPPORTED = -5
RB_E_RANGE = -6
RB_E_IO = -7

RC_NAMES = {
    -1: "unsupported shape",
    -2: "shape not tileable",
    -3: "allocation failed",
    -4: "device/driver failure",
    -5: "unsupported feature",
    -6: "value out of range",
    -7: "argument/state failure",
}

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

MASK_NONE = 0
MASK_NONE_BLOCK = 1
MASK_CAUSAL = 2
MASK_WINDOW = 3
MASK_CAUSAL_WINDOW = 4
MASK_WINDOW_BLOCK = 5
MASK_CAUSAL_BLOCK = 6

WEIGHT_Q8_0 = 1
WEIGHT_W8A8 = 2

_i = C.c_int
_i64 = C.c_int64
_p = C.c_void_p
_f = C.c_float

# name -> (restype, argtypes)
TILES_AUTO, TILES_SINGLE, TILES_PAIR = 0, 1, 2

WEIGHT_I8G = 3
WEIGHT_F16 = 4

SIGNATURES = {
    "rb_init": (_i, [_i]),
    "rb_last_error": (_i, [C.c_char_p, C.c_size_t]),
    "rb_check_device_errors": (_i, []),
    "rb_pack_q8_0": (_i64, [_p, _i64, _i64]),
    "rb_pack_f32_q8_0": (_i64, [C.POINTER(_p), C.POINTER(_i64), _i, _i64]),
    "rb_pack_w8a8": (_i64, [_p, _p, _i64, _i64, _f, _f]),
    "rb_weight_info": (_i, [_i64, C.POINTER(_i), C.POINTER(_i64), C.POINTER(_i64)]),
    "rb_matmul": (_i, [_i64, _p, _i, _i64, _i64, _p, _i, _p]),
    "rb_matmul_host": (_i, [_i64, _p, _i, _i64, _i64, _p, _i]),
    "rb_matmul_w8a8_noalloc": (_i, [_i64, _p, _i, _i64, _i64, _p, _i, _p]),
    "rb_attention": (_i, [_p, _p, _p, _p, _i, _i64, _i64, _i, _i, _i, _f, _f, _i, _i64, _i64, _i64, _p]),
    "rb_attention_host": (_i, [_p, _p, _p, _p, _i, _i64, _i64, _i, _i, _i, _f, _f, _i, _i64, _i64, _i64]),
    "rb_pack_f32_q8_0_device": (_i64, [C.POINTER(_p), C.POINTER(_i64), _i, _i64]),
    "rb_attention_batched": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _i64, _i64, _i64, _i, _i, _i, _f, _f,
                                  _i, _i64, _i64, _i64, _p]),
    "rb_rms_norm": (_i, [_p, _i, _p, _f, _p, _i, _i64, _i64, _p]),
    "rb_pack_f32_w8a8_device": (_i64, [_p, _i64, _i64, _f, _f]),
    "rb_pack_i8": (_i64, [_p, _i64, _i64, _i64]),
    "rb_pack_f16": (_i64, [_p, _p, _i, _i64, _i]),
    "rb_quantize_row_groups": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _p]),
    "rb_add_layer_norm": (_i, [_p, _p, _p, _p, _f, _p, _i64, _i64, _p]),
    "rb_gelu": (_i, [_p, _i64, _p]),
    "rb_silu_mul": (_i, [_p, _p, _i, _p, _i64, _p]),
    "rb_gelu_mul": (_i, [_p, _p, _i, _p, _i64, _p]),
    "rb_rope": (_i, [_p, _i, _p, _p, _p, _i64, _i64, _i, _i, _p]),
    "rb_embed_gather": (_i, [_p, _i64, _p, _i64, _i64, _p, _p]),
    "rb_add_rms_norm": (_i, [_p, _p, _p, _f, _p, _i64, _i64, _p]),
    "rb_qk_norm_rope": (_i, [_p, _i64, _i64, _i, _i, _i, _p, _p, _f, _p, _p, _i64, _p]),
    "rb_silu_mul_halves": (_i, [_p, _i64, _i64, _p, _p]),
    "rb_last_token_l2": (_i, [_p, _i64, _i64, _i64, _p, _f, _p, _p]),
    "rb_q8_0_dequant": (_i, [_i64, _p, _i, _p]),
    "rb_quantize_rows_i8": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "rb_matmul_i8_acc": (_i, [_i64, _p, _i64, _p, _p]),
    "rb_mem_stats": (_i, [C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]),
    "rb_launch_count": (_i64, [_i]),
    "rb_set_tile_policy": (_i, [_i]),
    "rb_set_attention_split": (_i, [_i]),
    "rb_matmul_w8a8_codes": (_i, [_i64, _p, _p, _i64, _i64, _p, _i, _p]),
    "rb_add_layer_norm_quant": (_i, [_p, _p, _p, _p, _f, _p, _p, _i64, _i64, _p]),
    "rb_set_weight_activation": (_i, [_i64, _i]),
    "rb_pack_f32_q8_0_gated_device": (_i64, [_p, _p, _i64, _i64]),
    "rb_selftest_wait_timeout": (_i, [_i64, _p]),
    "rb_moe_workspace_bytes": (_i64, [_i64, _i, _i]),
    "rb_moe_max_rows": (_i64, [_i64, _i, _i]),
    "rb_moe_slot_rows_offset": (_i64, [_i64, _i, _i]),
    "rb_moe_route": (_i, [_p, _i64, _i, _i, _i, _p, _p, _p]),
    "rb_moe_dispatch": (_i, [_p, _i64, _i, _i, _p, _i64, _p, _p, _p]),
    "rb_matmul_grouped": (_i, [_i64, _i, _p, _i64, _p, _i64, _i, _p, _i, _p]),
    "rb_moe_combine": (_i, [_p, _p, _i64, _p, _p, _p, _i64, _i, _i, _p]),
    "rb_ep_build_send": (_i, [_p, _i64, _i, _i, _i, _p, _i64, _p, _p, _p, _p, _p, _p]),
    "rb_ep_build_send_capacity": (_i, [_p, _i64, _i, _i, _i, _i64, _p, _i64, _p, _p, _p, _p, _p, _p]),
    "rb_gather_rows": (_i, [_p, _p, _i64, _i64, _p, _p]),
    "rb_moe_combine_rows": (_i, [_p, _p, _i64, _p, _p, _p, _i64, _i, _p]),
}

_lib = None


def load(path: os.PathLike | str | None = None) -> C.CDLL:
    """Load (once) and return the library with its signatures declared."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m burn_rocket_b200.build` "
            "(librocket_b200 has no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().rb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")
