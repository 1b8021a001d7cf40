"""Shared pytest setup: the `gpu` marker, repository imports, and helpers.

`-m "not gpu"` tests run anywhere (no CUDA device needed); `-m gpu` tests need
a B200 and call the engine through its C ABI (libnsfps.so) or its pybind11
module.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def yf():
    """The drop-in module (fails loudly when the extension is not built)."""
    from ns_fps_b200 import yuezu_fps_module
    return yuezu_fps_module


@pytest.fixture(scope="session")
def capi():
    from tests import capi as c
    return c


def reference_dir():
    """The reference checkout when this machine has one (never the GPU box):
    $NSFPS_REFERENCE_DIR, else BASELINE.json's reference_path; None when
    absent."""
    import json
    ref = os.environ.get("NSFPS_REFERENCE_DIR")
    if not ref:
        try:
            with open(os.path.join(ROOT, "BASELINE.json")) as f:
                ref = json.load(f).get("reference_path")
        except (OSError, ValueError):
            ref = None
    return ref if ref and os.path.isdir(ref) else None
