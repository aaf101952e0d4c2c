import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def ctx():
    """A libocb context on cuda:0 (GPU tests only)."""
    from opencuda import api
    c = api.Context(0)
    yield c
    c.close()
