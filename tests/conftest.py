"""Shared pytest configuration.

Markers: ``gpu`` — needs a CUDA device (B200); everything else runs on CPU.
The native module is imported from the source tree (built in place).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def has_gpu():
    import torch

    return torch.cuda.is_available()


@pytest.fixture
def lo_env(monkeypatch):
    """Loopback fabric for the MPComm objects created in a test."""
    monkeypatch.setenv("MPCOMM_FABRIC", "lo")
    monkeypatch.setenv("MPCOMM_LOG_LEVEL", "1")
    yield
