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
def g_qe8():
    return load_golden("golden_qe8.npz")


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


def same_bits_or_nan(a, b):
    """same_bits, except that a NaN matches any NaN: IEEE 754 leaves the sign
    and payload of a generated NaN (inf * 0) to the hardware (x86 SSE gives
    0xFFC00000, the GPU 0x7FFFFFFF)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb)) and same_bits(a[~na], b[~nb])


def qe8_same_or_tie(got, ref, A, bpw, group=256, max_ties=4):
    """q_e8 outputs (qlab.py:185-198) bit-equal except on 8-vectors whose two
    reconstructions are codewords at exactly equal distance from gn (checked
    in rational arithmetic) -- ties that cKDTree breaks by the order of its
    tree search.  Returns the number of tied vectors (at most max_ties)."""
    from fractions import Fraction
    import oracle as O
    got = np.ascontiguousarray(got, np.float64).ravel()
    ref = np.ascontiguousarray(ref, np.float64).ravel()
    if got.shape != ref.shape:
        return -1
    diff = np.flatnonzero(got.view(np.int64) != ref.view(np.int64))
    if diff.size == 0:
        return 0
    cb = O.e8_codebook(1 << int(round(bpw * 8)))
    flat = np.asarray(A, np.float64).ravel()
    flat = np.concatenate([flat, np.zeros((-flat.size) % group)])
    g = flat.reshape(-1, group)
    s = np.repeat(np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12, group, axis=1).reshape(-1, 8)
    gn = (g / (np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12)).reshape(-1, 8)
    vecs = np.unique(diff // 8)
    assert vecs.size <= max_ties, f"{vecs.size} vectors differ"
    n = got.size
    for v in vecs:
        valid = np.arange(8 * v, min(8 * v + 8, n)) - 8 * v
        def code(out):
            rec = cb * s[v][None, :]
            hit = np.all(rec[:, valid].view(np.int64) == out[8 * v + valid].view(np.int64)[None, :], axis=1)
            j = np.flatnonzero(hit)
            assert j.size, f"vector {v}: output is not a scaled codeword"
            return int(j[0])
        jg, jr = code(got), code(ref)
        exact = [sum((Fraction(float(gn[v, i])) - Fraction(float(cb[j, i]))) ** 2 for i in range(8)) for j in (jg, jr)]
        assert exact[0] == exact[1], f"vector {v}: codewords {jg} and {jr} are not at equal distance"
        d = ((gn[v][None, :] - cb) ** 2).sum(1)
        assert float(exact[0]) <= d.min() * (1 + 1e-12), f"vector {v}: not a nearest codeword"
    return int(vecs.size)


def near_tie_codebook(L, seed):
    """A codebook of 2^L float32 entries that are four base values each
    moved by at most 3 * 2^-22 relative: the candidate costs of a Viterbi
    step then lie within a few ulps of one another, so a cost formed with a
    single rounding instead of the reference's two (a contracted
    multiply-add) changes the chosen path on many sequences."""
    rng = np.random.RandomState(seed)
    base = rng.randn(4).astype(np.float32)
    pert = rng.randint(-3, 4, size=1 << L).astype(np.float32)
    return (base[np.arange(1 << L) % 4] * (1 + pert * np.float32(2 ** -22))).astype(np.float32)
