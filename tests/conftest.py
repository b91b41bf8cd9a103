"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU.

The oracle (oracle/) is the checker for every parity test; it is built here
if its shared object is missing.  The product library is never replaced by
the oracle: GPU tests call libhexatrain_b200.so through its C ABI.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU case")


def _cuda_device_count() -> int:
    try:
        import ctypes
        lib = ctypes.CDLL("libcuda.so.1")
        if lib.cuInit(0) != 0:
            return 0
        n = ctypes.c_int(0)
        if lib.cuDeviceGetCount(ctypes.byref(n)) != 0:
            return 0
        return n.value
    except OSError:
        return 0


HAS_GPU = _cuda_device_count() > 0


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build
    build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("reference CPU build (oracle/_ref) not present")
    return Reference()


@pytest.fixture(scope="session")
def gpu_runtime():
    import hexatrain_b200 as hx
    rt = hx.Runtime()
    assert rt.initialize(0), rt.last_error
    yield rt
    rt.close()


def golden(name):
    data = np.load(os.path.join(GOLDEN, name))
    return {k: data[k] for k in data.files}


def rel_err(got, want) -> float:
    """max |got - want| / max |want|  (tensor-wise relative error)."""
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    assert g.shape == w.shape, (g.shape, w.shape)
    den = max(float(np.max(np.abs(w))) if w.size else 0.0, 1e-30)
    return float(np.max(np.abs(g - w))) / den if w.size else 0.0
