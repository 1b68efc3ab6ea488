import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu)")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    if not O.LIB.exists():
        O.build(with_reference=False)
    return O


@pytest.fixture(scope="session")
def reference(oracle_mod):
    if not oracle_mod.Reference.available():
        pytest.skip("PyFlame reference shim not built (oracle/_ref)")
    return oracle_mod.Reference()


@pytest.fixture(scope="session")
def native():
    from pyflame_b200 import _native
    if not _native.LIB_PATH.exists():
        from pyflame_b200 import build
        build.build()
    return _native


@pytest.fixture(scope="session")
def cuda_executor(native):
    from pyflame_b200.backend import CudaExecutor, cuda_is_available
    if not cuda_is_available():
        pytest.fail("GPU test collected but no sm_100 GPU is visible")
    ex = CudaExecutor(CudaExecutor.Config())
    yield ex
    ex.close()


@pytest.fixture
def rng():
    return np.random.default_rng(42)


@pytest.fixture(autouse=True)
def fresh_graph():
    import pyflame_b200 as pf
    pf.reset_graph()
    yield
