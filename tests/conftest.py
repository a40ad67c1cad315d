"""Shared test setup: import paths, the `gpu` marker, checker and library fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "compressed-kv-attention_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    if not os.path.exists(O.ORACLE_SO):
        O.build()
    return O.oracle()


@pytest.fixture(scope="session")
def reference():
    """The compiled reference library, or skip when oracle/_ref was not built."""
    import oracle as O
    r = O.reference()
    if r is None:
        pytest.skip("reference library (oracle/_ref) not built on this host")
    return r


@pytest.fixture(scope="session")
def reference_or_none():
    """The compiled reference library when oracle/_ref was built here, else None."""
    import oracle as O
    return O.reference()


@pytest.fixture(scope="session")
def kvx():
    import build
    build.build()
    import kvexp_b200
    return kvexp_b200


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
