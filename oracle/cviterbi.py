"""ctypes loader of the C restatement of the segmented Viterbi
(``uq_viterbi_ref.c``): TEST INFRASTRUCTURE ONLY, like the rest of oracle/.

The C file follows trellis.py:84-105 operation for operation (float32 sub,
multiply, add; first index on ties) and is checked against the numpy / torch
restatement ``uq_oracle.viterbi_segments`` and the reference goldens by
``tests/test_oracle_golden.py``.  It exists because the torch restatement
runs L = 16 at about 10 k weights/s, too slow to check whole tensors.

``build()`` compiles it with gcc into ``oracle/_build/`` (it is rebuilt when
the source is newer than the library).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "uq_viterbi_ref.c")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(OUT, "libuq_viterbi_ref.so")
# -ffp-contract=off: no fused multiply-add (the reference rounds the square
# and the sum separately); no fast-math
CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared"]

_lock = threading.Lock()
_lib = None


def build() -> str:
    os.makedirs(OUT, exist_ok=True)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    tmp = LIB + f".{os.getpid()}.tmp"
    r = subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gcc failed for {SRC}:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def load() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            lib = ctypes.CDLL(build())
            lib.uq_oracle_viterbi.restype = ctypes.c_int
            lib.uq_oracle_viterbi.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
            lib.uq_oracle_viterbi_fused.restype = ctypes.c_int
            lib.uq_oracle_viterbi_fused.argtypes = lib.uq_oracle_viterbi.argtypes
            lib.uq_oracle_path_cost.restype = ctypes.c_float
            lib.uq_oracle_path_cost.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
            _lib = lib
        return _lib


def viterbi_segments_c(xn, L: int, R: int, cw=None, threads: int = 0, fused: bool = False) -> np.ndarray:
    """Same contract as ``uq_oracle.viterbi_segments`` (int64 states, (nseq, T)).
    ``fused=True`` forms each cost with one fused multiply-add instead of the
    reference's two roundings: not the reference, only a probe that finds
    the sequences on which contraction changes the path."""
    from .uq_oracle import codebook
    x = np.ascontiguousarray(xn, np.float32)
    if x.ndim != 2:
        raise ValueError("xn must be (nseq, T)")
    c = np.ascontiguousarray(codebook(L) if cw is None else cw, np.float32)
    out = np.empty(x.shape, np.int32)
    fn = load().uq_oracle_viterbi_fused if fused else load().uq_oracle_viterbi
    rc = fn(x.ctypes.data, x.shape[0], x.shape[1], L, R, c.ctypes.data, out.ctypes.data, int(threads))
    if rc != 0:
        raise RuntimeError("uq_oracle_viterbi failed")
    return out.astype(np.int64)


def path_costs(xn, states, L: int, cw=None) -> np.ndarray:
    """fp32 cost of each row's state path under the Viterbi recurrence."""
    from .uq_oracle import codebook
    x = np.ascontiguousarray(xn, np.float32)
    st = np.ascontiguousarray(states, np.int32)
    c = np.ascontiguousarray(codebook(L) if cw is None else cw, np.float32)
    lib = load()
    T = x.shape[1]
    return np.array([lib.uq_oracle_path_cost(x[i].ctypes.data, st[i].ctypes.data, T, c.ctypes.data)
                     for i in range(x.shape[0])], np.float32)
