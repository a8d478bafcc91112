"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs everywhere (oracle vs golden fixtures, host logic, the C ABI's exports and
argument validation); `-m gpu` runs the parity tests of the CUDA kernels on a B200.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "flb-transformer_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    import torch
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


@pytest.fixture(scope="session")
def attn_golden():
    return load_golden("attention.pt")


@pytest.fixture(scope="session")
def wf_golden():
    return load_golden("wavefront.pt")


@pytest.fixture(scope="session")
def flb_golden():
    return load_golden("flb_model.pt")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
