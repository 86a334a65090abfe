"""Shared pytest configuration: the `gpu` marker and common fixtures."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a engine)")


def _has_gpu() -> bool:
    try:
        from vicinity_b200 import device_count

        return device_count() > 0
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if any("gpu" in it.keywords for it in items) and not _has_gpu():
        skip = pytest.mark.skip(reason="no CUDA device visible")
        for it in items:
            if "gpu" in it.keywords:
                it.add_marker(skip)


@pytest.fixture(scope="session")
def kats():
    return json.loads((GOLDEN / "reference_kats.json").read_text())
