import sys
from pathlib import Path

import pytest

TESTS = Path(__file__).resolve().parent
ROOT = TESTS.parent
for p in (str(TESTS), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu on the GPU box)")


@pytest.fixture(scope="session")
def oracle():
    from oracle_ffi import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ctx():
    import adi_b200
    context = adi_b200.Context(0)
    # The tests stage inputs and outputs with torch on the default stream:
    # the context launches there too, so the two stay ordered.
    context.set_stream(adi_b200.CUDA_STREAM_LEGACY)
    yield context
    context.close()
