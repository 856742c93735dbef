"""Shared pytest configuration.

``gpu``-marked tests need a B200 and the built CUDA library; everything else
runs on CPU.
"""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def golden_dir():
    return REPO / "tests" / "golden"
