"""Test configuration: import paths, the `gpu` marker, in-tree native builds."""

import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "mlvc.cpp_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session", autouse=True)
def native_builds():
    """Builds the oracle library and the product library when sources changed."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "oracle"], check=True)
    import build  # mlvc.cpp_b200/build.py
    build.build()
