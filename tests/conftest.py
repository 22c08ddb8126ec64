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


def group_loss_case(fixture, case: str):
    """``(windows, slots, positions)`` of one case of ``golden/group_loss.npz``:
    ``windows`` as ``(anchor, labels)`` pairs, ``slots`` None for the model's
    default block, ``positions`` the per-position label weights or None."""
    labels = fixture[f"{case}_labels"].tolist()
    windows, at = [], 0
    for anchor, length in zip(fixture[f"{case}_anchors"].tolist(), fixture[f"{case}_lengths"].tolist()):
        windows.append((anchor, tuple(labels[at:at + length])))
        at += length
    slots = int(fixture[f"{case}_slots"])
    positions = tuple(fixture[f"{case}_positions"].tolist()) if f"{case}_positions" in fixture.files else None
    return tuple(windows), (None if slots < 0 else slots), positions
