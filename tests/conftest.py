"""Shared pytest setup.

`-m gpu` tests need a B200 and call the library through its C ABI;
everything else runs on the CPU (oracle vs golden fixtures, host logic, ABI
loading and argument checks, gloo multi-rank merge logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", os.path.join("metal-flat_b200", "python")):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (run with -m gpu)")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="session")
def built_lib():
    """Build the in-tree libraries once if they are missing (CPU-side compile)."""
    import mflat_b200
    if not os.path.exists(mflat_b200.LIB_PATH):
        import subprocess
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "metal-flat_b200")], check=True)
    return mflat_b200.lib()
