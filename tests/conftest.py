import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG = os.path.join(ROOT, "lightining-core_b200")
for p in (ROOT, os.path.join(PKG, "python")):
    if p not in sys.path:
        sys.path.insert(0, p)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def golden(name):
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def close_enough(ref, got, atol, rtol):
    """tests/test_backend_parity.cpp:25-63 of the reference: |a-b| <= atol + rtol*|ref| everywhere."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    assert ref.shape == got.shape, (ref.shape, got.shape)
    err = np.abs(ref - got)
    bad = err > atol + rtol * np.abs(ref)
    if bad.any():
        i = int(np.argmax(err))
        raise AssertionError(f"mismatch at flat {i}: ref={ref.flat[i]} got={got.flat[i]} "
                             f"max_abs={err.max():.3g} n_bad={int(bad.sum())} (atol={atol}, rtol={rtol})")
    return float(err.max()) if err.size else 0.0


@pytest.fixture(scope="session")
def lc():
    import lightning_core_b200 as m
    return m


@pytest.fixture(scope="session")
def gpu(lc):
    if not lc.cuda_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return lc
