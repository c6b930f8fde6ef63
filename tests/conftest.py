"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200) and the built
libpagedattn.so; everything else runs on CPU.  Parity tests compare the CUDA
path against the numpy oracle in ``oracle/`` and the committed golden vectors
in ``tests/golden/`` (made from the reference by tests/golden/make_golden.py).
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built libpagedattn.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test ran without a CUDA device")
    from mini_llm_runtime_b200 import _lib

    _lib.load()  # fails loudly if the library is missing
    return torch.device("cuda", 0)
