"""Shared pytest configuration: the ``gpu`` marker and import helpers."""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PACKAGE = "binary-eagle-decoding_b200"


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def package():
    """The product package (its directory name is not a Python identifier)."""
    return importlib.import_module(PACKAGE)


def submodule(name: str):
    return importlib.import_module(f"{PACKAGE}.{name}")


@pytest.fixture(scope="session")
def bd():
    return package()
