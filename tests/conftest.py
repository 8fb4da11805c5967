import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")
    config.addinivalue_line("markers", "slow: full-size workload (minutes)")


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ctx():
    """One library context on cuda:0 for the GPU tests."""
    if not _cuda_ok():
        pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
    from voxcpm_rs_b200.minicpm4 import Context
    c = Context(0)
    yield c
    c.close()


def assert_close(got, want, atol, rtol, what=""):
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got - want)
    tol = atol + rtol * np.abs(want)
    bad = err > tol
    if bad.any():
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} elements out of tolerance "
                             f"(atol={atol}, rtol={rtol}); worst at {i}: got {got[i]}, want {want[i]}, "
                             f"max abs err {err.max():.3e}")
