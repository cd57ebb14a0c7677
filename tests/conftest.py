import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(__file__))

import _oracle  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def port():
    return _oracle.Port()


@pytest.fixture(scope="session")
def ref():
    if not _oracle.ensure_ref():
        pytest.skip("reference oracle library not built (oracle/_ref) and reference sources absent")
    return _oracle.Ref(_oracle.REF_AVX2)


@pytest.fixture(scope="session")
def ref_scalar():
    if not _oracle.ensure_ref():
        pytest.skip("reference oracle library not built (oracle/_ref) and reference sources absent")
    return _oracle.Ref(_oracle.REF_SCALAR)


@pytest.fixture(scope="session")
def pkg():
    return _oracle.load_pkg()


@pytest.fixture(scope="session")
def gpu(pkg):
    """The CUDA C ABI bound to cuda:0 (GPU tests only)."""
    pkg.init(0)
    yield pkg
    pkg.shutdown()
