"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle/golden, ABI-surface and host-logic tests on any
machine; `-m gpu` runs the device parity tests through the C ABI on a B200.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and librocket_b200.so")


@pytest.fixture(scope="session")
def rb():
    """The product package, initialised on cuda:0 (GPU tests only)."""
    import torch
    import burn_rocket_b200 as rb_mod
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    rb_mod.init(0)
    return rb_mod


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as orc_mod
    orc_mod.lib()
    return orc_mod
