import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def ctx():
    """One kk_ctx for the whole GPU session."""
    import kokopop_b200 as kb
    c = kb.Context(0)
    yield c
    c.close()
