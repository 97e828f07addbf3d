"""Drop-in replacement for UltraQuant's ``trellis.py`` (trellis.py:14-108).

``codebook``, ``pred_table``, ``trellis_quant`` and ``trellis_quant_fast``
keep the reference signatures and return the same float32 arrays; the
normalisation, Viterbi search and decoding run in libuq_b200.  The
``device`` argument is accepted for compatibility: work always runs on the
current CUDA device (or on ``device`` when it names a CUDA device).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _device as D
from . import _lib

__all__ = ["codebook", "pred_table", "trellis_quant", "trellis_quant_fast", "encode_segments",
           "viterbi_states"]


def _dev(device) -> torch.device:
    if isinstance(device, (str, torch.device)) and str(device).startswith("cuda"):
        d = torch.device(device)
        if d.index is None:
            d = D.device()
        return d
    return D.device()


def codebook(L, seed=0):
    """trellis.py:14-19 -- float32 Gaussian codebook of 2^L hashed states
    (``seed`` is unused, as in the reference)."""
    del seed
    return D.to_host(D.codebook(int(L)))


def pred_table(L, R):
    """trellis.py:21-25 -- predecessor states (2^L, 2^R) int64."""
    S = 1 << L
    s = np.arange(S)[:, None]
    k = np.arange(1 << R)[None, :]
    return ((s >> R) | (k << (L - R))) & (S - 1)


def viterbi_states(xn: torch.Tensor, L: int, R: int, cw: torch.Tensor | None = None) -> torch.Tensor:
    """Min-plus Viterbi over the rows of ``xn`` (nseq, T) float32 CUDA tensor;
    returns the int32 state path (nseq, T)."""
    lib = _lib.load()
    nseq, T = xn.shape
    cw = D.codebook(L, xn.device) if cw is None else cw
    states = torch.empty((nseq, T), dtype=torch.int32, device=xn.device)
    if nseq:
        nbytes = lib.uq_trellis_workspace_bytes(nseq, T, L, R)
        if nbytes == 0:
            _lib.check(lib.uq_trellis_viterbi(None, nseq, T, L, R, None, None, None, 0, None), "viterbi")
        ws = D.workspace(nbytes, xn.device)
        _lib.check(lib.uq_trellis_viterbi(xn.data_ptr(), nseq, T, L, R, cw.data_ptr(), states.data_ptr(),
                                          ws.data_ptr(), ws.numel(), D.stream_handle(xn.device)), "viterbi")
        if L == 16:  # the cluster-split kernel reports bounded-wait timeouts
            _lib.check(lib.uq_device_errors(D.stream_handle(xn.device)), "viterbi")
    return states


def encode_segments(a: torch.Tensor, L: int, R: int, seg: int, scale_group: int):
    """Flat normalisation + Viterbi of trellis.py:69-103 on a CUDA tensor.
    Returns (states (Nseg, seg) int32, sc_g (G,) float32, ntot, pad)."""
    lib = _lib.load()
    ntot = a.numel()
    pad = (-ntot) % scale_group
    padded = ntot + pad
    if padded % seg:
        raise ValueError(f"cannot reshape array of size {padded} into shape (-1, {seg})")
    xn = torch.empty(padded, dtype=torch.float32, device=a.device)
    sc = torch.empty(padded // scale_group, dtype=torch.float32, device=a.device)
    st = D.stream_handle(a.device)
    if padded:
        _lib.check(lib.uq_trellis_normalize(a.data_ptr(), D.dtype_code(a), ntot, scale_group, seg,
                                            xn.data_ptr(), sc.data_ptr(), st), "normalize")
    states = viterbi_states(xn.view(-1, seg), L, R)
    return states, sc, ntot, pad


def trellis_quant_fast(A, L=12, R=2, seg=64, scale_group=256, mem_gb=3.0, device="cuda"):
    """trellis.py:62-108 -- segmented Viterbi, returns cw[s] * sc_g (float32)."""
    del mem_gb  # the library batches backpointers by its own workspace bound
    lib = _lib.load()
    dev = _dev(device)
    a = D.as_device(A, dev=dev)
    nrow, ncol = a.shape
    states, sc, ntot, _ = encode_segments(a, L, R, seg, scale_group)
    cw = D.codebook(L, dev)
    out = torch.empty((nrow, ncol), dtype=torch.float32, device=dev)
    if ntot:
        _lib.check(lib.uq_trellis_decode(states.data_ptr(), cw.data_ptr(), sc.data_ptr(), scale_group, ntot,
                                         out.data_ptr(), D.stream_handle(dev)), "decode")
    return out if isinstance(A, torch.Tensor) and A.is_cuda else D.to_host(out)


def trellis_quant(A, L=10, R=2, group=256, chunk_rows=512, device="cuda"):
    """trellis.py:27-60 -- full-row Viterbi (one sequence per padded row)."""
    del chunk_rows
    lib = _lib.load()
    dev = _dev(device)
    a = D.as_device(A, dev=dev)
    nrow, T = a.shape
    Tp = ((T + group - 1) // group) * group
    xn = torch.empty((nrow, Tp), dtype=torch.float32, device=dev)
    sc = torch.empty((nrow, Tp // group), dtype=torch.float32, device=dev)
    st = D.stream_handle(dev)
    out = torch.empty((nrow, T), dtype=torch.float32, device=dev)
    if nrow and T:
        _lib.check(lib.uq_trellis_normalize_rows(a.data_ptr(), D.dtype_code(a), nrow, T, T, group,
                                                 xn.data_ptr(), sc.data_ptr(), st), "normalize_rows")
        states = viterbi_states(xn, L, R)
        cw = D.codebook(L, dev)
        _lib.check(lib.uq_trellis_decode_rows(states.data_ptr(), cw.data_ptr(), sc.data_ptr(), nrow, T, Tp,
                                              group, out.data_ptr(), st), "decode_rows")
    return out if isinstance(A, torch.Tensor) and A.is_cuda else D.to_host(out)
