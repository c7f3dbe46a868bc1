import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def ref_lib():
    """The reference compiled from its sources (oracle/_ref); skips when it is not built."""
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref/libveda_ref.so not built (make -C oracle)")
    return ref


@pytest.fixture(scope="session")
def cuda():
    """The product library (CUDA kernels behind the C ABI) on cuda:0."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import veda_b200
    return veda_b200.lib()
