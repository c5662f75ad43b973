import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs through libsheafb200 on cuda:0)")


@pytest.fixture(scope="session")
def lib():
    from sheaf_b200 import build, session
    build.build()
    return session.library()


@pytest.fixture(scope="session")
def fp32_session(lib):
    from sheaf_b200.session import B200Session
    s = B200Session(device=0, precision="fp32")
    yield s
    s.close()


@pytest.fixture(scope="session")
def tf32_session(lib):
    from sheaf_b200.session import B200Session
    s = B200Session(device=0, precision="tf32")
    yield s
    s.close()


@pytest.fixture(scope="session")
def bf16_session(lib):
    from sheaf_b200.session import B200Session
    s = B200Session(device=0, precision="bf16")
    yield s
    s.close()
