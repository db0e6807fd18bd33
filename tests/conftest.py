"""Shared pytest configuration.

``gpu``-marked tests need a B200 (sm_100a) and the in-tree CUDA library; all
other tests run on the CPU (oracle checks, host logic, C-ABI symbol checks).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built libaoscuda.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o
