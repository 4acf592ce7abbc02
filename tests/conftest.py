import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def native_lib():
    from leanstream_b200 import build

    if build.needs_build():
        try:
            build.build()
        except RuntimeError as exc:  # pragma: no cover - nvcc always exists in this image
            pytest.fail(f"native library build failed: {exc}")
    from leanstream_b200 import _native

    return _native.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail("the sm_100a library needs a B200-class (sm_100) device")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
