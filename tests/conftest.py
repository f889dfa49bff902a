"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked gpu need a B200 and the built libcatsgpu.so; everything else runs
on the CPU (oracle vs golden fixtures, host logic, library exports).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libcatsgpu.so")


@pytest.fixture(scope="session")
def orc():
    from oracle.cpu import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref_llm():
    from oracle.cpu import Reference, ref_available
    if not ref_available("llm"):
        pytest.skip("compiled reference (oracle/_ref) not built here")
    return Reference("llm")


@pytest.fixture(scope="session")
def ref_cnn():
    from oracle.cpu import Reference, ref_available
    if not ref_available("cnn"):
        pytest.skip("compiled reference (oracle/_ref) not built here")
    return Reference("cnn")


@pytest.fixture(scope="session")
def gpu():
    """Initialise libcatsgpu on cuda:0 (fails, not skips, when the library is missing)."""
    from catseye_b200 import _lib
    return _lib.init(0)
