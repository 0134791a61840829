"""Test setup: package paths, the `gpu` marker, and shared helpers."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "qwen-native-engine_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) and runs the CUDA kernels")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major < 10:
        pytest.fail("these kernels are built for sm_100a (B200)")
    return torch.device("cuda:0")
