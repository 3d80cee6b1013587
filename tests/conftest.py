"""Shared pytest setup.

`gpu` marks tests that need a B200; everything else runs on the CPU.
The package directory is named `pico-sglang_b200`, so it is imported with
importlib and exposed to tests through the `pgb` fixture and `load_pgb()`.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

os.environ.setdefault("MASTER_ADDR", "127.0.0.1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


def load_pgb():
    return importlib.import_module("pico-sglang_b200")


@pytest.fixture(scope="session")
def pgb():
    return load_pgb()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    return torch.device("cuda", 0)
