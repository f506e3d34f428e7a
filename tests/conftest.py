"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (sm_100) and the built library; the rest run on
any CPU host and never launch a kernel.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
