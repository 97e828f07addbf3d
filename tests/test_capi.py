"""The C-ABI library loads and exports every entry point of include/uq_b200.h
(no compute calls: this runs without a GPU), plus host-only entry points."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "uq_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(uq_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from ultraquant_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from ultraquant_b200 import build
        build.build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    from ultraquant_b200 import _lib
    assert set(names) == set(_lib.SIGNATURES), "ctypes prototypes must mirror the header"


def test_status_strings(lib):
    assert lib.uq_status_string(0) == b"ok"
    assert lib.uq_version() >= 100


def test_next_pow2(lib):
    import oracle as O
    for n in [0, 1, 2, 3, 5, 300, 4096, 4097, 14336, 28672]:
        assert lib.uq_next_pow2(n) == O.next_pow2(n)


def test_signs_match_numpy_mt19937(lib, g_rht):
    for n in [1, 2, 64, 1024, 32768]:
        out = np.empty(n, np.float64)
        assert lib.uq_rht_signs(0, n, out.ctypes.data) == 0
        assert np.array_equal(out.astype(np.int8), g_rht[f"signs_{n}"])
    out = np.empty(1024, np.float64)
    lib.uq_rht_signs(7, 1024, out.ctypes.data)
    assert np.array_equal(out.astype(np.int8), g_rht["signs_seed7_1024"])
    for seed in (1, 12345, 2**32 - 1):
        o = np.empty(5000, np.float64)
        lib.uq_rht_signs(seed, 5000, o.ctypes.data)
        assert np.array_equal(o, np.random.RandomState(seed).choice([-1.0, 1.0], size=5000))


def test_argument_validation_without_gpu(lib):
    # invalid shapes are rejected before any device work
    assert lib.uq_rht_rows(None, 1, 4, 0, 0, None, None, None) == 1
    assert lib.uq_trellis_viterbi(None, 4, 64, 17, 2, None, None, None, 0, None) == 2
    assert lib.uq_trellis_viterbi(None, 4, 64, 8, 5, None, None, None, 0, None) == 2
    assert lib.uq_trellis_normalize(None, 0, 300, 256, 64, None, None, None) == 1  # 512 % 64 ok but null ptr
    assert lib.uq_trellis_normalize(None, 0, 300, 256, 384, None, None, None) == 1  # 512 % 384 != 0
    assert b"seg" in lib.uq_last_error()
    assert lib.uq_e8_quant(None, 1, 10, 12, 0.5, None, None, None) == 2          # group % 8
    assert lib.uq_trellis_workspace_bytes(100, 256, 16, 2) > 100 * 255 * 1024 * 4 // 2
    assert lib.uq_trellis_workspace_bytes(100, 256, 17, 2) == 0


def test_workspace_queries(lib):
    assert lib.uq_quant_trellis_workspace_bytes(4096, 4096, 16, 2, 256, 256) > 4096 * 4096 * 4
    assert lib.uq_quant_e8_workspace_bytes(4096, 14336, 256) >= 4096 * 16384 * 8
    assert lib.uq_e8_entropy_workspace_bytes(600000) > 600000 * 8
