import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA backend)")
    config.addinivalue_line("markers", "slow: full-size parity case (seconds of CPU oracle time)")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def gpu_ctx_factory():
    from tensor_logic_lang_b200.runtime import Context

    def make(**kw):
        return Context(**kw)
    return make
