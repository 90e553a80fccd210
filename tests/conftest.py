"""Test configuration: the ``gpu`` marker, import paths and shared fixtures.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic, the
C-ABI library loads and exports its symbols, multi-process ``gloo`` tests).
``-m gpu`` needs a B200 and fails loudly -- never skips -- when the CUDA
library or the device is missing.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden():
    d = os.path.join(ROOT, "tests", "golden")
    return {n: np.load(os.path.join(d, n + ".npz")) for n in ("gating", "quant", "routing")}


@pytest.fixture(scope="session")
def cuda():
    """The torch CUDA device after checking the library is the native one."""
    import torch
    import aethermoe_b200 as aem
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    aem.lib()  # raises if libaethermoe.so is missing
    if aem.device_count() < 1:
        pytest.fail("no sm_100 (B200) device visible to libaethermoe")
    return torch.device("cuda", 0)
