"""Drop-in replacement for the hot-path functions of UltraQuant's ``qlab.py``.

Same names, arguments, dtypes and results as the reference (qlab.py:53-183);
the arithmetic runs in libuq_b200 on the GPU.  Functions accept host numpy
arrays (returning numpy, like the reference) or CUDA tensors (returning CUDA
tensors, no host round trip).
"""
from __future__ import annotations

import ctypes

import numpy as np

import torch

from . import _device as D
from . import _lib
from .q8 import deq_q8  # noqa: F401  (qlab.py:27-32, used by load_WH)

__all__ = ["wnmse", "_next_pow2", "rht_rows", "irht_rows", "_d8_decode", "e8_decode",
           "_entropy_bpw", "q_e8_fast", "_E8_SCALE", "deq_q8", "q_uniform", "e8_codebook", "q_e8",
           "e8_scale_search"]

# qlab.py:158 -- calibrated E8 step per calib_key, reused across tensors
_E8_SCALE: dict = {}


def _is_dev(a) -> bool:
    return isinstance(a, torch.Tensor) and a.is_cuda


def _ret(t: torch.Tensor, like):
    """Result in the caller's form, after checking that no bounded device
    wait of the tensor-map kernels timed out (that would leave ``t`` wrong;
    the check synchronises the stream, as the host copy does anyway)."""
    _lib.check(_lib.load().uq_device_errors(D.stream_handle(t.device)), "qlab")
    return t if _is_dev(like) else D.to_host(t)


def wnmse(A, Ah) -> float:
    """qlab.py:53-54 -- sum((A - Ah)^2) / sum(A^2), both sums in fp64 on the
    device (fixed-order reduction; numpy's pairwise order differs, ~1e-15)."""
    lib = _lib.load()
    a = D.as_device(A)
    b = D.as_device(Ah, dev=a.device)
    if a.shape != b.shape:
        raise ValueError(f"operands could not be broadcast together with shapes {tuple(a.shape)} {tuple(b.shape)}")
    if a.dtype not in (torch.float32, torch.float64):
        a = a.to(torch.float64)
    if b.dtype not in (torch.float32, torch.float64):
        b = b.to(torch.float64)
    out = torch.empty(2, dtype=torch.float64, device=a.device)
    ws = D.workspace(lib.uq_wnmse_workspace_bytes(), a.device)
    _lib.check(lib.uq_wnmse_sums(a.data_ptr() if a.numel() else None, D.dtype_code(a),
                                 b.data_ptr() if b.numel() else None, D.dtype_code(b), a.numel(),
                                 out.data_ptr(), ws.data_ptr(), ws.numel(), D.stream_handle(a.device)), "wnmse")
    e = D.to_host(out)
    with np.errstate(divide="ignore", invalid="ignore"):
        return float(e[0] / e[1])


def _next_pow2(n: int) -> int:
    """qlab.py:66-69."""
    return int(_lib.load().uq_next_pow2(int(n)))


def _signs_n(n: int, seed: int, dev):
    return D.signs(n, seed, dev)


def rht_rows(A, seed=0, block28=False):
    """qlab.py:71-85 -- randomized Hadamard transform along rows (fp64 out).
    ``block28=True`` (opt-in, no reference counterpart) uses the unpadded
    H_28 (x) H_P transform for widths 28 x 512 and 28 x 1024."""
    lib = _lib.load()
    a = D.as_device(A)
    if a.dim() != 2:
        raise ValueError("rht_rows expects a 2-D array (out, in)")
    rows, n0 = a.shape
    if block28:
        out = torch.empty((rows, n0), dtype=torch.float64, device=a.device)
        if rows:
            d = _signs_n(n0, seed, a.device)
            _lib.check(lib.uq_rht28_rows(a.data_ptr(), D.dtype_code(a), rows, n0, n0, None, d.data_ptr(),
                                         out.data_ptr(), D.stream_handle(a.device)), "rht_rows(block28)")
        return _ret(out, A)
    if n0 == 0:  # the reference pads to one zero column
        a = torch.zeros((rows, 1), dtype=torch.float64, device=a.device)
        n0 = 1
    n = _next_pow2(n0)
    out = torch.empty((rows, n), dtype=torch.float64, device=a.device)
    if rows:
        d = D.signs(n, seed, a.device)
        _lib.check(lib.uq_rht_rows(a.data_ptr(), D.dtype_code(a), rows, n0, n0, d.data_ptr(),
                                   out.data_ptr(), D.stream_handle(a.device)), "rht_rows")
    return _ret(out, A)


def irht_rows(X, n0, seed=0, block28=False):
    """qlab.py:87-98 -- inverse of rht_rows, cropped to n0 columns (fp64).
    ``block28=True``: inverse of the opt-in unpadded transform (n0 = width)."""
    lib = _lib.load()
    x = D.as_device(X)
    rows, n = x.shape
    if block28:
        out = torch.empty((rows, n), dtype=torch.float64, device=x.device)
        if rows:
            d = _signs_n(n, seed, x.device)
            _lib.check(lib.uq_irht28_rows(x.data_ptr(), D.dtype_code(x), rows, n, n, None, d.data_ptr(),
                                          out.data_ptr(), 1, n, D.stream_handle(x.device)), "irht_rows(block28)")
        return _ret(out, X)
    if n & (n - 1):
        raise ValueError("irht_rows: width must be a power of two")
    n0 = int(n0)
    out = torch.empty((rows, min(n0, n)), dtype=torch.float64, device=x.device)
    if rows and n0:
        d = D.signs(n, seed, x.device)
        _lib.check(lib.uq_irht_rows(x.data_ptr(), D.dtype_code(x), rows, n, n, min(n0, n), d.data_ptr(),
                                    out.data_ptr(), D.stream_handle(x.device)), "irht_rows")
    return _ret(out, X)


def q_uniform(A, bpw, bs=32):
    """qlab.py:100-106 -- per-block absmax uniform quantizer (dtype of A)."""
    lib = _lib.load()
    a = D.as_device(A)
    lvl = (1 << (int(round(bpw)) - 1)) - 1
    out = torch.empty_like(a)
    if a.numel() % bs:
        raise ValueError(f"cannot reshape array of size {a.numel()} into shape (-1,{bs})")
    _lib.check(lib.uq_q_uniform(a.data_ptr() if a.numel() else None, D.dtype_code(a), a.numel(), int(bs), lvl,
                                out.data_ptr() if out.numel() else None, D.stream_handle(a.device)), "q_uniform")
    return _ret(out, A)


# qlab.py:110 -- codebooks per K (host fp64), and their device copies
_E8_CACHE: dict = {}
_E8_DEV: dict = {}


def _e8_grid_norms():
    """Lattice norms of the reference's point list (qlab.py:113-118): the
    grid g in [-3, 3]^8 (first coordinate slowest) with an even coordinate
    sum, then the same points plus 1/2.  |g|^2 and |g + 1/2|^2 = |g|^2 +
    sum(g) + 2 are integers, so the fp64 values equal the reference's
    (pts**2).sum(1) exactly.  Returns (grid ids of the even points, norms)."""
    v = np.arange(-3, 4, dtype=np.int64)
    sq, tot = v * v, v.copy()
    for _ in range(7):
        sq = np.add.outer(sq, v * v).ravel()
        tot = np.add.outer(tot, v).ravel()
    even = np.flatnonzero((tot & 1) == 0)
    n_int = sq[even]
    return even, np.concatenate([n_int, n_int + tot[even] + 2]).astype(np.float64)


def _e8_build(K):
    """(codebook, scale c, boundary norm) of qlab.py:111-124 for K points: the
    K points of smallest norm (np.argsort over the same norm list, so the
    members of the boundary shell are the reference's), each divided by
    c = sqrt(mean |p|^2 / 8); every grid point of lattice norm below the
    boundary norm is a codeword (+inf when K covers the grid)."""
    if K not in _E8_CACHE:
        even, norms = _e8_grid_norms()
        order = np.argsort(norms)
        ids = order[:K]
        ne = even.size
        gid = even[ids % ne]
        digits = (gid[:, None] // (7 ** np.arange(7, -1, -1, dtype=np.int64))) % 7
        pts = (digits - 3).astype(np.float64) + np.where(ids >= ne, 0.5, 0.0)[:, None]
        scale = np.sqrt((pts ** 2).sum(1).mean() / 8)
        cut = float(norms[order[K - 1]]) if K < norms.size else float("inf")
        _E8_CACHE[K] = (pts / scale, float(scale), cut)
    return _E8_CACHE[K]


def e8_codebook(K):
    """qlab.py:111-124 -- the (K, 8) fp64 codebook, bit for bit."""
    return _e8_build(K)[0]


def _e8_codebook_dev(K, dev):
    """Device copies (fp64, fp32) of e8_codebook(K), its scale and boundary norm."""
    key = (int(K), dev.index)
    if key not in _E8_DEV:
        cb, scale, cut = _e8_build(K)
        t64 = torch.from_numpy(np.ascontiguousarray(cb)).to(dev)
        _E8_DEV[key] = (t64, t64.to(torch.float32), scale, cut)
    return _E8_DEV[key]


def q_e8(A, bpw, group_scale=256):
    """qlab.py:185-198 -- per-group scaled 8-vectors to the nearest codeword of
    e8_codebook(2^round(8 bpw)) (fp64, A's shape).  Nearest as cKDTree's exact
    Euclidean query; on an exact fp64 distance tie the lowest index."""
    lib = _lib.load()
    K = 1 << int(round(bpw * 8))
    a = D.as_device(A)
    if a.dtype not in (torch.float32, torch.float64):
        a = a.to(torch.float64)
    out = torch.empty(tuple(a.shape), dtype=torch.float64, device=a.device)
    n = a.numel()
    if n:
        cb, cb32, scale, cut = _e8_codebook_dev(K, a.device)
        ws = D.workspace(lib.uq_q_e8_workspace_bytes(n, int(group_scale)), a.device)
        _lib.check(lib.uq_q_e8(a.data_ptr(), D.dtype_code(a), n, int(group_scale), cb.data_ptr(), cb32.data_ptr(),
                               cb.shape[0], scale, cut, out.data_ptr(), ws.data_ptr(), ws.numel(),
                               D.stream_handle(a.device)), "q_e8")
    return _ret(out, A)


def _d8_decode(Y):
    """qlab.py:133-142."""
    lib = _lib.load()
    y = D.as_device(Y, torch.float64).reshape(-1, 8)
    out = torch.empty_like(y)
    _lib.check(lib.uq_d8_decode(y.data_ptr(), y.shape[0], out.data_ptr(), D.stream_handle(y.device)), "_d8_decode")
    return _ret(out, Y)


def e8_decode(Y):
    """qlab.py:144-149."""
    lib = _lib.load()
    y = D.as_device(Y, torch.float64).reshape(-1, 8)
    out = torch.empty_like(y)
    _lib.check(lib.uq_e8_decode(y.data_ptr(), y.shape[0], out.data_ptr(), D.stream_handle(y.device)), "e8_decode")
    return _ret(out, Y)


def _entropy_bpw(idx_pts) -> float:
    """qlab.py:151-156 -- entropy of the distinct 8-tuples 2*pts, / 8."""
    lib = _lib.load()
    p = D.as_device(idx_pts, torch.float64).reshape(-1, 8)
    nvec = p.shape[0]
    ws = D.workspace(lib.uq_e8_entropy_workspace_bytes(nvec), p.device)
    res = torch.empty(1, dtype=torch.float64, device=p.device)
    _lib.check(lib.uq_e8_entropy_bpw(p.data_ptr(), nvec, res.data_ptr(), ws.data_ptr(), ws.numel(),
                                     D.stream_handle(p.device)), "_entropy_bpw")
    v = float(res.item())
    if v < 0:
        raise NotImplementedError("_entropy_bpw: a lattice index lies outside [-127, 127]")
    return v


def q_e8_fast(A, target_bpw=2.0, group=256, calib_key="g", fixed_step=None):
    """qlab.py:159-183 -- per-group RMS, one global step, E8 decode (fp64)."""
    lib = _lib.load()
    a = D.as_device(A)
    shape = tuple(a.shape)
    size = a.numel()
    st = D.stream_handle(a.device)
    if fixed_step is not None:
        step = float(fixed_step)
    else:
        if calib_key not in _E8_SCALE:
            ws = D.workspace(lib.uq_e8_calibrate_workspace_bytes(size, group), a.device)
            out = ctypes.c_double()
            _lib.check(lib.uq_e8_calibrate(a.data_ptr(), D.dtype_code(a), size, int(group), float(target_bpw),
                                           ctypes.addressof(out), ws.data_ptr(), ws.numel(), st),
                       "q_e8_fast calibration")
            _E8_SCALE[calib_key] = float(out.value)
        step = _E8_SCALE[calib_key]
    rec = torch.empty(shape, dtype=torch.float64, device=a.device)
    if size:
        _lib.check(lib.uq_e8_quant(a.data_ptr(), D.dtype_code(a), size, int(group), step, rec.data_ptr(), None, st),
                   "q_e8_fast")
    return _ret(rec, A)


def e8_scale_search(A, step, group=256):
    """Opt-in per-row scale search (no counterpart in the reference, whose
    q_e8_fast uses one global step, qlab.py:159-183): each row of the rotated
    matrix A (rows, n), n a multiple of 256, is quantized like
    q_e8_fast(fixed_step=s) at the one of 16 steps s = step * 2^((c-8)/8)
    picked by the rate-constrained search of uq_e8_scale_search.  Returns
    (rec fp64 like A, choice int32 per row, lam)."""
    if group != 256:
        raise ValueError("e8_scale_search quantizes groups of 256")
    lib = _lib.load()
    a = D.as_device(A, torch.float64)
    if a.dim() != 2:
        raise ValueError("e8_scale_search: A must be (rows, n)")
    rows, n = a.shape
    rec = torch.empty_like(a)
    choice = torch.empty(rows, dtype=torch.int32, device=a.device)
    lam = ctypes.c_double()
    ws = D.workspace(lib.uq_e8_scale_search_workspace_bytes(rows, n) if n >= 256 else 0, a.device)
    _lib.check(lib.uq_e8_scale_search(a.data_ptr(), rows, n, float(step), rec.data_ptr(), None, choice.data_ptr(),
                                      ctypes.addressof(lam), ws.data_ptr(), ws.numel(), D.stream_handle(a.device)),
               "e8_scale_search")
    if _is_dev(A):
        return rec, choice, float(lam.value)
    return D.to_host(rec), D.to_host(choice), float(lam.value)
