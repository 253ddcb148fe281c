"""Shared pytest configuration: markers and import paths.

`gpu` tests need a B200 and the built CUDA library; everything else runs on
the CPU (oracle pins, host logic, C-ABI export checks, gloo multi-rank logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "project-k3x_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and the built k3xb library")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def rs():
    from oracle import Restatement
    return Restatement()


@pytest.fixture(scope="session")
def ref():
    from oracle import Reference, have_reference
    if not have_reference():
        pytest.skip("oracle/_ref/libk3x_ref.so not built (reference tree absent)")
    return Reference()
