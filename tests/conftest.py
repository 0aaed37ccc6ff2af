"""Shared pytest configuration.

Marker `gpu`: the test needs a CUDA sm_100 device and runs the CUDA library
(parity tests proper). Everything else runs on the CPU.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100) and the CUDA library")


@pytest.fixture(scope="session")
def oracle():
    from oracle import pyoracle
    pyoracle.lib()
    return pyoracle


@pytest.fixture(scope="session")
def ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA")
    import ouroboros_b200 as oq
    c = oq.Context(0)
    yield c
    c.check_device()
    c.close()
