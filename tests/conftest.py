"""Test configuration: the `gpu` marker and import paths.

GPU tests call the product through lib/libdbs.so (C ABI) and the PyTorch
mirror; CPU tests cover the oracle against golden vectors, host-side logic and
the library's exported symbols.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "differentiable-beam-search-cuda_b200")
for p in (os.path.join(PKG, "python"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

LIBDBS = os.path.join(PKG, "lib", "libdbs.so")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libdbs.so")


@pytest.fixture(scope="session")
def libdbs():
    import dbs_ctypes
    return dbs_ctypes.load_library(LIBDBS)


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import OracleLib
    return OracleLib()
