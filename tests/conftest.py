import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built CUDA extension")
    config.addinivalue_line("markers", "slow: long-running test")
    # The host runtime is required by most tests; build it in-tree if it is missing.
    so = ROOT / "vm_c_b200" / "_ext" / "host" / "_host.so"
    if not so.exists():
        from vm_c_b200._build import build_host
        build_host()


@pytest.fixture(scope="session")
def host():
    from vm_c_b200 import _native
    return _native.host()


@pytest.fixture(scope="session")
def cuda_ext():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test needs CUDA")
    from vm_c_b200 import _native
    return _native.cuda()
