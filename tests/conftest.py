"""Shared fixtures.  `-m "not gpu"` runs on a CPU-only host; tests marked
`gpu` need a CUDA device and call the product library through its C ABI."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    return O.load_oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference's own kernels compiled through the NEON shim, or skip."""
    from oracle import oracle as O
    ref = O.load_reference()
    if ref is None:
        pytest.skip("oracle/_ref/libtinygiant_ref.so not built")
    return ref


@pytest.fixture(scope="session")
def lib():
    import tinygiant_b200 as tg
    return tg.load()


@pytest.fixture(scope="session")
def gpu(lib):
    """The product library on a GPU host; fails (not skips) if no device is
    visible, because gpu-marked tests only run where one must exist."""
    n = lib.tg_cuda_device_count()
    assert n > 0, "no CUDA device visible to libtinygiant.so"
    return lib


def golden(name):
    """Fixture arrays by name.  A dict (not the lazy NpzFile) so every lookup
    returns the same array object and pointers passed to C stay valid."""
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: np.ascontiguousarray(z[k]) for k in z.files}
