"""Shared test set-up. Tests marked `gpu` need a B200 and the built libvpass.so; everything else runs
on the CPU (the oracle against the reference's golden fixtures, host logic, the C ABI's exports)."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libvpass.so")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
