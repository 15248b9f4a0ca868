import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests are skipped (not failed) when no GPU is visible, so the CPU
    # suite can be run with or without ``-m "not gpu"``.
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture
def qkv_plan():
    """Set a QKV plan override for one test (``qkv_plan(impl=1, splits=3)``);
    the automatic plan is restored afterwards."""
    from flash_dllm_b200 import ops
    yield ops.set_qkv_plan
    ops.set_qkv_plan()
    ops.set_gemm_plan()
