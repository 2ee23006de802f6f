import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "vllm-factory_b200", ROOT / "tests" / "golden", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_error_word_clean(request):
    """Every GPU test must leave the kernels' device error word at zero: a bounded wait
    that ran out (a lost arrival, a pipeline mismatch) is a failure even when the
    output happens to be right."""
    yield
    if "gpu" not in request.keywords:
        return
    import torch
    if not torch.cuda.is_available():
        return
    import vf_b200
    torch.cuda.synchronize()
    word = vf_b200.device_error(clear=True)
    assert word == 0, f"device error word {word:#x} after {request.node.name}"
