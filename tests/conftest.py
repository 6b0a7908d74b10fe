"""Shared pytest setup: the `gpu` marker and import paths."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built engine")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def engine():
    """One engine on cuda:0 for the whole GPU session."""
    import emeans_b200

    e = emeans_b200.Engine(device=0)
    yield e
    e.close()
