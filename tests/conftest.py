"""Shared fixtures: the package (loaded by path), the CPU checkers, and the
`gpu` marker for tests that need a B200."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__ as entry  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def ufb():
    return entry.load_package()


@pytest.fixture(scope="session")
def syn():
    return entry.load_synthetic()


@pytest.fixture(scope="session")
def ora():
    import oracle
    return oracle.c_oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libufref.so not built")
    return oracle.ref_oracle()


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
