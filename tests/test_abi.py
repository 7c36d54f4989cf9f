"""C-ABI surface checks that need no GPU: the library loads, exports every
symbol include/rocket_b200.h declares, and reports the reference's status
codes for misuse before init (lib.rs:116-146)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "rocket_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^RB_API\s+[\w\s\*]+?\b(rb_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_surface():
    syms = declared_symbols()
    for must in ["rb_init", "rb_pack_q8_0", "rb_pack_f32_q8_0", "rb_pack_w8a8", "rb_matmul",
                 "rb_attention", "rb_last_error", "rb_mem_stats"]:
        assert must in syms


def test_library_exports_every_declared_symbol():
    from burn_rocket_b200 import _lib
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_codes_match_the_reference():
    from burn_rocket_b200 import _lib
    assert (_lib.RB_E_SHAPE, _lib.RB_E_TILING, _lib.RB_E_NOMEM, _lib.RB_E_DEVICE,
            _lib.RB_E_UNSUPPORTED, _lib.RB_E_RANGE, _lib.RB_E_IO) == (-1, -2, -3, -4, -5, -6, -7)
    text = HEADER.read_text()
    for name, val in [("RB_E_SHAPE", -1), ("RB_E_TILING", -2), ("RB_E_NOMEM", -3), ("RB_E_DEVICE", -4),
                      ("RB_E_UNSUPPORTED", -5), ("RB_E_RANGE", -6), ("RB_E_IO", -7)]:
        assert re.search(rf"#define {name} \({val}\)", text)


def test_calls_before_init_fail_with_io_status():
    from burn_rocket_b200 import _lib
    lib = _lib.load()
    buf = (C.c_float * 4)()
    assert lib.rb_matmul(1, C.addressof(buf), 0, 1, 4, C.addressof(buf), 0, None) == _lib.RB_E_IO
    assert "rb_init" in _lib.last_error()
    assert lib.rb_pack_w8a8(None, None, 32, 32, 0.0, 0.0) == _lib.RB_E_IO


def test_op_failure_payload():
    import burn_rocket_b200 as rb
    with pytest.raises(rb.OpFailure) as ei:
        rb._check(-2, "rocket_matmul", 4, 8, 16)
    e = ei.value
    assert e.error.rc == -2 and e.error.is_fallback() and (e.m, e.k, e.n) == (4, 8, 16)


def test_init_without_gpu_reports_device_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from burn_rocket_b200 import _lib
    rc = _lib.load().rb_init(0)
    assert rc == _lib.RB_E_DEVICE
