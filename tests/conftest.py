"""pytest configuration: the `gpu` marker and shared fixtures."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle_mod():
    from metalllm_b200.build import build_oracle
    build_oracle()
    from oracle import oracle
    oracle.load()
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import _lib
    return _lib.load()
