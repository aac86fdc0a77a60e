"""Shared pytest set-up.

`gpu` marks tests that need a B200; everything else runs on CPU.  The CPU
oracle (oracle/, test infrastructure) is built once per session.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o

    o.build()
    return o
