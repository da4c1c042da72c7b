import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def native_lib():
    """The C-ABI library, built in-tree first if it is missing or stale (nvcc cross-compiles)."""
    from qwen3_engine_from_scratch_b200 import _native, build
    if not os.path.exists(_native.LIB_PATH) or not build.up_to_date():
        try:
            build.build()
        except RuntimeError as e:  # no nvcc here and no prebuilt library
            pytest.skip(f"cannot build the native library: {e}")
    return _native.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
