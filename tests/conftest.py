"""Shared pytest setup.

Markers
  gpu   needs a CUDA sm_100 device (run with `-m gpu` on a B200 box; deselected on CPU).

GPU tests call the kernel through the C ABI (flash_attn_npu_b200/_native.py -> libfa_sm100.so)
and compare against the CPU/fp32 oracle in oracle/attention_ref.py.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an NVIDIA sm_100 (B200) GPU")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def native_lib():
    """Build (if needed) and load libfa_sm100.so."""
    from flash_attn_npu_b200 import build, _native
    if not build.LIB_PATH.exists() or os.environ.get("FA_REBUILD") == "1":
        build.build()
    return _native.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)
