import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running parity case")


def _ensure_built():
    from tinybrain_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from tinybrain_b200 import build
        build.build()
    import oracle
    if not os.path.exists(oracle.LIB_PATH):
        oracle.build()


_ensure_built()


@pytest.fixture(scope="session")
def ctx():
    from tinybrain_b200.runtime import Context, device_count
    if device_count() == 0:
        pytest.skip("no CUDA device")
    return Context.default(0)
