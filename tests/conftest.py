import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libmvr_b200.so")


@pytest.fixture(scope="session")
def orc():
    """The CPU parity oracle (built on first use)."""
    from oracle import oracle

    oracle.build()
    oracle.load()
    return oracle


@pytest.fixture(scope="session")
def ctx():
    """A library context on cuda:0. Fails (does not skip) without a GPU."""
    from ir_multivector_retrieval_b200 import Context

    c = Context(int(os.environ.get("MVR_DEVICE", "0")))
    yield c
    c.close()
