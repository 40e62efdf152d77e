import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def _isolate_env(monkeypatch):
    """Tests never inherit kernel-forcing or fault-injection settings from the caller."""
    for var in ("MTLFLASHATTN_KERNEL", "MFA_FAULT", "MTLFLASHATTN_TRACE", "MTLFLASHATTN_TORCH_CHUNK"):
        monkeypatch.delenv(var, raising=False)
    yield
