import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def g_rht():
    return load_golden("golden_rht.npz")


@pytest.fixture(scope="session")
def g_e8():
    return load_golden("golden_e8.npz")


@pytest.fixture(scope="session")
def g_trellis():
    return load_golden("golden_trellis.npz")


@pytest.fixture(scope="session")
def g_pipeline():
    return load_golden("golden_pipeline.npz")


@pytest.fixture(scope="session")
def g_quniform():
    return load_golden("golden_quniform.npz")


@pytest.fixture(scope="session")
def g_q8():
    return load_golden("golden_q8.npz")


@pytest.fixture(scope="session")
def g_qat():
    return load_golden("golden_qat.npz")


def qat_meta(g, key):
    vals = [int(v) for v in g[key + "_meta"]]
    meta = dict(zip(("nrow", "ncol", "Ntot", "seg", "scale_group", "pad", "Nseg"), vals[:7]))
    return meta, vals[7], vals[8]          # meta, L, in0


def grad_close(got, ref, exact, rtol=2e-6):
    """Gradient sums: |got - exact| within one fp32 rounding of the fp64 sum
    (plus rtol of the norm), and the reference's fp32-accumulated sums within
    rtol * ||exact|| as well."""
    got, ref, exact = (np.asarray(v, np.float64) for v in (got, ref, exact))
    scale = np.abs(exact).max() + 1e-30
    ok_got = np.all(np.abs(got - exact) <= np.abs(exact) * 2 ** -23 + rtol * scale)
    ok_ref = np.all(np.abs(ref - exact) <= 1e-4 * scale)
    return bool(ok_got and ok_ref)


def same_bits(a, b):
    """Bit-for-bit equality of two float arrays (signed zeros included)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    iv = {4: np.int32, 8: np.int64, 2: np.int16, 1: np.int8}[a.dtype.itemsize]
    return bool(np.array_equal(a.view(iv), b.view(iv)))
