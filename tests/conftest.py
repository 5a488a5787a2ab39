"""Test configuration: the `gpu` marker (tests that need a B200; run with -m gpu) and shared fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as O
    return O.Oracle()


@pytest.fixture
def decode_only():
    """Keeps every call of the test on the decode kernels (prefill threshold above any T), then restores it."""
    import mvcc_b200 as m
    m.set_prefill_min_tokens(1 << 30)
    yield
    m.set_prefill_min_tokens(0)
