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


def pytest_terminal_summary(terminalreporter):
    """Prints how many tokens the GPU parity tests left out of their value comparisons (near 8th/9th routing ties)."""
    from tests import parity
    if not parity.EXCLUDED:
        return
    tot = sum(n for _, _, n, _ in parity.EXCLUDED)
    out = sum(x for _, x, _, _ in parity.EXCLUDED)
    tr = terminalreporter
    tr.write_sep("-", "parity: tokens left out near routing ties")
    tr.write_line(f"{len(parity.EXCLUDED)} comparisons, {out} of {tot} tokens left out, smallest 8th/9th margin "
                  f"{min(m for _, _, _, m in parity.EXCLUDED):.3g}")
    for name, x, n, m in parity.EXCLUDED:
        if x:
            tr.write_line(f"  {name}: {x} of {n} left out (smallest margin {m:.3g})")
