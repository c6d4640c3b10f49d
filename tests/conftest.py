import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libaexis_cuda on cuda:0)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # oracle/oracle.py (test infrastructure)
    O.build()
    return O


@pytest.fixture(scope="session")
def ops():
    import torch
    from aiimage_b200.ops import AexisOps
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    o = AexisOps(0)
    yield o
    torch.cuda.synchronize()
    o.close()
