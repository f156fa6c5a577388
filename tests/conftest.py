"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked `gpu` need a B200 (sm_100) and call the CUDA kernels through the
C ABI of libpfng_b200.  Everything else runs on the CPU: the oracle against
the golden fixtures and the reference, the host-side argument checks of the
C ABI, and multi-process (gloo) sharding logic.
"""
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT / "qgemm-perf-framework-ng_b200"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle_lib import reference_or_none
    ref = reference_or_none()
    if ref is None:
        pytest.skip("reference checker (oracle/_ref) not built here; golden fixtures pin the oracle instead")
    return ref


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(ROOT / "tests" / "golden" / "golden.npz"))
