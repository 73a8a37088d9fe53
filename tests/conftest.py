import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen3-vl_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)



def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running")
    config.addinivalue_line(
        "markers", "gpu_pending: parity tests of kernels that have not yet had their first "
        "GPU run; they run only with Q3VL_PENDING_GPU_TESTS=1")


def pytest_collection_modifyitems(config, items):
    pending = os.environ.get("Q3VL_PENDING_GPU_TESTS") == "1"
    skip_pending = pytest.mark.skip(reason="kernels awaiting their first GPU run "
                                           "(set Q3VL_PENDING_GPU_TESTS=1)")
    for it in items:
        if "gpu_pending" in it.keywords and not pending:
            it.add_marker(skip_pending)
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
