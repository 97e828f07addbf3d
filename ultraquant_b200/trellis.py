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
           "viterbi_states", "packed_words", "pack_states", "unpack_states"]


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


# ---------------------------------------------------------------------------
# Packed codes (the L + R (T-1) bits per sequence behind the reference's
# bits-per-weight accounting of qat.trellis_encode's state paths)
# ---------------------------------------------------------------------------
def packed_words(T: int, L: int, R: int) -> int:
    """32-bit words per packed sequence of T states."""
    return int(_lib.load().uq_trellis_packed_words(int(T), int(L), int(R)))


def pack_states(states, L: int, R: int):
    """(nseq, T) int32 state paths -> (nseq, packed_words) uint32 bit strings
    S = s_0 2^(R(T-1)) + sum_t (s_t mod 2^R) 2^(R(T-1-t)), low word first.
    numpy in -> numpy out; CUDA tensors in -> CUDA tensors out."""
    lib = _lib.load()
    on_dev = isinstance(states, torch.Tensor) and states.is_cuda
    st = states if on_dev else torch.from_numpy(np.ascontiguousarray(np.asarray(states, dtype=np.int32)))
    st = st.to(D.device() if not on_dev else st.device).to(torch.int32).contiguous()
    nseq, T = st.shape
    words = packed_words(T, L, R)
    if words == 0:
        raise ValueError(f"pack_states: unsupported T={T} L={L} R={R}")
    out = torch.empty((nseq, words), dtype=torch.int32, device=st.device)
    _lib.check(lib.uq_trellis_pack(st.data_ptr(), nseq, T, L, R, out.data_ptr(), D.stream_handle(st.device)),
               "pack_states")
    return out if on_dev else D.to_host(out).view(np.uint32)


def unpack_states(packed, T: int, L: int, R: int):
    """Inverse of pack_states: (nseq, packed_words) -> (nseq, T) int32."""
    lib = _lib.load()
    on_dev = isinstance(packed, torch.Tensor) and packed.is_cuda
    pk = packed if on_dev else torch.from_numpy(np.ascontiguousarray(np.asarray(packed).view(np.int32)))
    pk = pk.to(D.device() if not on_dev else pk.device).contiguous()
    nseq = pk.shape[0]
    if pk.shape[1] != packed_words(T, L, R):
        raise ValueError(f"unpack_states: {pk.shape[1]} words per sequence, expected {packed_words(T, L, R)}")
    out = torch.empty((nseq, T), dtype=torch.int32, device=pk.device)
    _lib.check(lib.uq_trellis_unpack(pk.data_ptr(), nseq, T, L, R, out.data_ptr(), D.stream_handle(pk.device)),
               "unpack_states")
    return out if on_dev else D.to_host(out)
