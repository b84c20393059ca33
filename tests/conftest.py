"""Test configuration: the ``gpu`` marker and repo-root imports.

``-m "not gpu"`` runs the CPU suite (oracle vs golden vectors, C-ABI symbol
table, host logic, gloo multi-rank logic); ``-m gpu`` runs the CUDA parity
tests, which call the product through torch.ops.d2p / the C ABI and compare
against the CPU oracle in ``oracle/`` (test infrastructure only).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch

    return torch.device("cuda:0")
