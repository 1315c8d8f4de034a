"""Shared pytest setup: the ``gpu`` marker, import paths and package loader."""

from __future__ import annotations

import importlib
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PACKAGE_NAME = "gpu-kernel-for-transformer_b200"
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library"
    )


def load_package():
    """Import the package, whose directory name is not a Python identifier."""
    return importlib.import_module(PACKAGE_NAME)


@pytest.fixture(scope="session")
def pkg():
    return load_package()


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.pt"))


def load_golden(name):
    import torch

    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)
