"""Test configuration: the `gpu` marker, import paths and shared fixtures.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's known
values, the host-side logic and the C ABI's exports.  GPU tests (`-m gpu`)
compare the CUDA engine, called through the C ABI, with the oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "forge-db_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and runs the CUDA engine")


@pytest.fixture(scope="session")
def ctx():
    import forgegpu as fg
    return fg.default_context()


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle
