"""Drop-in replacement for the encoder and the differentiable decoder of
UltraQuant's ``qat.py`` (qat.py:11-59).

* ``trellis_encode`` returns the reference's tuple
  ``(states (Nseg, seg) int32, sc_g (G, 1) float32, cw (2^L,) float32, meta)``.
* ``fwht_torch``, ``irht_torch`` and ``recon_torch`` are autograd functions
  whose forward and backward run in libuq_b200 (``uq_fwht``,
  ``uq_qat_recon``, ``uq_qat_recon_backward``).  Forward values are the
  reference's bit for bit; gradients agree with torch's to fp32 rounding of
  the two sums (the kernels accumulate them in fp64).  ``recon_torch``
  differentiates with respect to ``cw`` and ``sc_g`` (the QAT parameters,
  qat.py:70-72); ``sH`` is a constant.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _device as D
from . import _lib
from .trellis import encode_segments

__all__ = ["DEV", "trellis_encode", "fwht_torch", "irht_torch", "recon_torch"]

DEV = "cuda"


def trellis_encode(A, L=12, R=2, seg=64, scale_group=256):
    """qat.py:11-33 -- the segmented Viterbi of trellis_quant_fast, returning
    the state path instead of the reconstruction."""
    a = D.as_device(A)
    nrow, ncol = a.shape
    states, sc, ntot, pad = encode_segments(a, L, R, seg, scale_group)
    meta = dict(nrow=nrow, ncol=ncol, Ntot=ntot, seg=seg, scale_group=scale_group, pad=pad,
                Nseg=states.shape[0])
    return (D.to_host(states), D.to_host(sc).reshape(-1, 1).astype(np.float32),
            D.to_host(D.codebook(L, a.device)), meta)


# ---------------------------------------------------------------------------
# FWHT / inverse RHT (qat.py:35-49)
# ---------------------------------------------------------------------------
def _float_dtype(t: torch.Tensor) -> None:
    if t.dtype not in (torch.float32, torch.float64):
        raise NotImplementedError(f"fwht: dtype {t.dtype} is not built (float32 / float64)")


def _fwht_call(x2d: torch.Tensor, n: int, signs, colscale, direction: int, ncols_out: int) -> torch.Tensor:
    """x2d: contiguous CUDA (rows, ncols_in) -> (rows, ncols_out) in x2d's dtype."""
    lib = _lib.load()
    rows, ncols_in = x2d.shape
    out = torch.empty((rows, ncols_out), dtype=x2d.dtype, device=x2d.device)
    _lib.check(lib.uq_fwht(x2d.data_ptr() if x2d.numel() else None, D.dtype_code(x2d), rows, n, max(ncols_in, 1),
                           ncols_in, D.ptr(signs), D.ptr(colscale), direction, out.data_ptr() if out.numel() else None,
                           max(ncols_out, 1), ncols_out, D.stream_handle(x2d.device)), "fwht")
    return out


def _signs_like(n: int, seed: int, like: torch.Tensor) -> torch.Tensor:
    return D.signs(n, seed, like.device).to(like.dtype)


class _Fwht(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, signs, ncols_out):
        n = x.shape[-1]
        ctx.n, ctx.ncols_in = n, n
        ctx.save_for_backward(signs)
        y = _fwht_call(x.reshape(-1, n).contiguous(), n, signs, None, 0, ncols_out)
        return y.reshape(*x.shape[:-1], ncols_out)

    @staticmethod
    def backward(ctx, g):
        (signs,) = ctx.saved_tensors
        k = g.shape[-1]
        gx = _fwht_call(g.reshape(-1, k).contiguous(), ctx.n, signs, None, 1, ctx.n)
        return gx.reshape(*g.shape[:-1], ctx.n), None, None


def _on_device(x: torch.Tensor):
    """CUDA view of x and a function restoring x's device on the result."""
    if x.is_cuda:
        return x, (lambda y: y)
    home = x.device
    return x.to(D.device()), (lambda y: y.to(home))


def fwht_torch(x):
    """qat.py:35-41 -- fast Walsh-Hadamard transform along the last axis
    (n = 2^k), normalised by 1/sqrt(n); differentiable."""
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(np.asarray(x))
    _float_dtype(x)
    n = x.shape[-1]
    if n & (n - 1) or n == 0:
        raise RuntimeError(f"fwht_torch: last dimension {n} is not a power of two")
    xd, back = _on_device(x)
    return back(_Fwht.apply(xd, None, n))


def irht_torch(Xrot, in0, seed=0):
    """qat.py:43-49 -- differentiable inverse of qlab.rht_rows:
    (fwht_torch(Xrot) * d)[:, :in0] with d the RandomState(seed) signs."""
    if not isinstance(Xrot, torch.Tensor):
        Xrot = torch.as_tensor(np.asarray(Xrot))
    _float_dtype(Xrot)
    out, n = Xrot.shape
    if n & (n - 1) or n == 0:
        raise RuntimeError(f"irht_torch: width {n} is not a power of two")
    in0 = len(range(n)[:int(in0)])          # Python slice semantics of [:, :in0]
    xd, back = _on_device(Xrot)
    return back(_Fwht.apply(xd, _signs_like(n, seed, xd), in0))


# ---------------------------------------------------------------------------
# recon_torch (qat.py:51-59)
# ---------------------------------------------------------------------------
def _states_device(states, dev) -> torch.Tensor:
    if isinstance(states, torch.Tensor):
        t = states
        if t.dtype not in (torch.int32, torch.int64):
            t = t.to(torch.int64)
    else:
        arr = np.asarray(states)
        if arr.dtype not in (np.int32, np.int64):
            arr = arr.astype(np.int64)
        t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.to(dev).contiguous().reshape(-1)


class _Recon(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cw, sc, st, signs, sH, nrow, n, group, in0):
        lib = _lib.load()
        out = torch.empty((nrow, in0), dtype=torch.float32, device=cw.device)
        _lib.check(lib.uq_qat_recon(st.data_ptr(), int(st.dtype == torch.int64), nrow, n, cw.data_ptr(),
                                    cw.numel(), sc.data_ptr(), group, signs.data_ptr(), D.ptr(sH), in0,
                                    out.data_ptr(), max(in0, 1), D.stream_handle(cw.device)), "recon_torch")
        ctx.save_for_backward(cw, sc, st, signs, sH)
        ctx.shape = (nrow, n, group, in0)
        return out

    @staticmethod
    def backward(ctx, g):
        cw, sc, st, signs, sH = ctx.saved_tensors
        nrow, n, group, in0 = ctx.shape
        lib = _lib.load()
        g = g.to(torch.float32).contiguous()
        gcw = torch.empty_like(cw)
        gsc = torch.empty_like(sc)
        nbytes = lib.uq_qat_recon_backward_workspace_bytes(cw.numel(), sc.numel())
        ws = D.workspace(nbytes, cw.device)
        _lib.check(lib.uq_qat_recon_backward(g.data_ptr(), max(in0, 1), st.data_ptr(), int(st.dtype == torch.int64),
                                             nrow, n, cw.data_ptr(), cw.numel(), sc.data_ptr(), sc.numel(), group,
                                             signs.data_ptr(), D.ptr(sH), in0, gcw.data_ptr(), gsc.data_ptr(),
                                             ws.data_ptr(), ws.numel(), D.stream_handle(cw.device)),
                   "recon_torch backward")
        return gcw, gsc, None, None, None, None, None, None, None


def recon_torch(states, cw, sc_g, meta, sH, in0):
    """qat.py:51-59 -- differentiable What = irht_torch(cw[states] * sc_g) / sH
    from fixed states and learnable (cw, sc_g); returns (nrow, in0) float32."""
    dev = cw.device if isinstance(cw, torch.Tensor) and cw.is_cuda else D.device()
    cw_t = cw if isinstance(cw, torch.Tensor) else torch.as_tensor(np.asarray(cw))
    sc_t = sc_g if isinstance(sc_g, torch.Tensor) else torch.as_tensor(np.asarray(sc_g))
    if cw_t.dtype != torch.float32 or sc_t.dtype != torch.float32:
        raise NotImplementedError("recon_torch: cw and sc_g must be float32 (the encoder's dtype)")
    nrow, ncol, ntot = int(meta["nrow"]), int(meta["ncol"]), int(meta["Ntot"])
    group, nseg, seg = int(meta["scale_group"]), int(meta["Nseg"]), int(meta["seg"])
    if ncol & (ncol - 1) or ncol == 0:
        raise RuntimeError(f"recon_torch: width {ncol} is not a power of two")
    if nrow * ncol != ntot:
        raise RuntimeError(f"recon_torch: shape '[{nrow}, {ncol}]' is invalid for input of size {ntot}")
    st = _states_device(states, dev)
    if st.numel() < nseg * seg or (nseg * seg) % group or sc_t.numel() != nseg * seg // group:
        raise RuntimeError("recon_torch: states / sc_g do not match meta "
                           f"({st.numel()} states, {sc_t.numel()} scales, Nseg*seg={nseg * seg}, group={group})")
    if isinstance(states, np.ndarray) and states.size:
        lo, hi = int(states.min()), int(states.max())
        if lo < 0 or hi >= cw_t.numel():
            raise IndexError(f"recon_torch: state {hi if hi >= cw_t.numel() else lo} is out of bounds "
                             f"for a codebook of {cw_t.numel()}")
    in0 = len(range(ncol)[:int(in0)])
    if sH is None:
        sH_t = None
    else:
        sH_t = sH if isinstance(sH, torch.Tensor) else torch.as_tensor(np.asarray(sH))
        if sH_t.dtype != torch.float32:
            raise NotImplementedError("recon_torch: sH must be float32 (qat.py:69)")
        sH_t = sH_t.detach().to(dev).reshape(-1)
        if sH_t.numel() == 1:
            sH_t = sH_t.expand(in0)
        if sH_t.numel() != in0:
            raise RuntimeError(f"recon_torch: sH has {sH_t.numel()} values for {in0} columns")
        sH_t = sH_t.contiguous()
    cw_d = cw_t if cw_t.device == dev else cw_t.to(dev)
    sc_d = (sc_t if sc_t.device == dev else sc_t.to(dev)).reshape(-1)
    signs = _signs_like(ncol, 0, cw_d)
    return _Recon.apply(cw_d.contiguous(), sc_d.contiguous(), st, signs, sH_t, nrow, ncol, group, in0)
