"""Shared pytest setup: import paths, the ``gpu`` marker, the package handle."""

from __future__ import annotations

import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
for p in (REPO, TESTS, os.path.join(TESTS, "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

PACKAGE = "quantized-llm-inference-engine-_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """Import the product package (its directory name is not an identifier)."""
    return importlib.import_module(PACKAGE)


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def lib(pkg):
    """The loaded C-ABI library (ctypes handle)."""
    return pkg.lib()


@pytest.fixture(scope="session")
def cuda():
    if not cuda_available():
        pytest.skip("no CUDA device")
    import torch

    return torch.device("cuda", 0)


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


__all__ = ["REPO", "PACKAGE", "load_package", "cuda_available"]
_ = os.environ
