import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "dream-tts_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def tt():
    """The ttsnn package with its CUDA library loaded (GPU tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    import ttsnn
    from ttsnn import _lib
    _lib.load()
    return ttsnn
