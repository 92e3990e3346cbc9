import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "ds-experiment_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "ds_ref_vectors.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def dso():
    from oracle import dso as _dso
    _dso.build()
    return _dso


def assert_bits_equal(got, want, what=""):
    """Bit-exact comparison; NaNs must line up (payloads are not compared)."""
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert got.dtype == want.dtype, (what, got.dtype, want.dtype)
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), f"{what}: NaN positions differ ({int((gn != wn).sum())})"
    itype = {4: np.uint32, 8: np.uint64}[got.dtype.itemsize]
    gb = got.view(itype)[~gn]
    wb = want.view(itype)[~wn]
    bad = np.nonzero(gb != wb)[0]
    assert bad.size == 0, (
        f"{what}: {bad.size} of {gb.size} differ; first at {bad[0]}: "
        f"got {got[~gn][bad[0]]!r} want {want[~wn][bad[0]]!r}")
