import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "torch-pyodide_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def cuda_rt():
    from tpcuda import CudaRuntime
    return CudaRuntime()


@pytest.fixture(scope="session")
def oracle_rt():
    from oracle_runtime import OracleRuntime
    return OracleRuntime()
