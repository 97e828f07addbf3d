"""Importance-weighted builder recipes on the fused device path.

``quant_trellis`` is buildtrellis.py:16-20 and ``quant_step`` is
buildalloc.py:21-24: clamp the imatrix, whiten ``A = W * sqrt(H)``, rotate,
quantize, rotate back, un-whiten.  One C-ABI call each
(``uq_quant_trellis`` / ``uq_quant_e8``); intermediates stay on the device.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _device as D
from . import _lib

__all__ = ["quant_trellis", "quant_step", "QuantResult", "quant_trellis_device", "quant_step_device"]


@dataclass
class QuantResult:
    What: torch.Tensor            # (rows, n0) float32
    err: torch.Tensor             # [sum (A - Ah)^2, sum A^2] fp64
    states: torch.Tensor | None = None   # (Nseg, seg) int32 (trellis)
    sc: torch.Tensor | None = None       # (G,) float32 (trellis)
    idx: torch.Tensor | None = None      # (rows * n,) int16 (E8, 2 * lattice point)
    choice: torch.Tensor | None = None   # (rows,) int32 candidate step per row (E8 scale search)
    lam: float | None = None             # rate multiplier of the scale search

    @property
    def wnmse(self) -> float:
        e = self.err.double().cpu()
        return float(e[0] / e[1])


def _device_status(lib, dev, what):
    """Raise if a bounded device wait of the kernels just launched gave up
    (their outputs would be wrong).  Synchronises the stream."""
    _lib.check(lib.uq_device_errors(D.stream_handle(dev)), what)


def quant_trellis_device(W: torch.Tensor, H: torch.Tensor, L=12, R=2, seg=64, scale_group=256, seed=0,
                         keep_codes=True, check_errors=True) -> QuantResult:
    """Device-resident buildtrellis recipe (W float32/float64, H float64).
    ``check_errors``: after the launch, synchronise and raise UQError if a
    bounded device wait timed out (their results would be wrong)."""
    lib = _lib.load()
    dev = W.device
    rows, n0 = W.shape
    n = int(lib.uq_next_pow2(n0))
    H = H.to(device=dev, dtype=torch.float64).contiguous()
    W = W.contiguous()
    cw = D.codebook(L, dev)
    d = D.signs(n, seed, dev)
    What = torch.empty((rows, n0), dtype=torch.float32, device=dev)
    # the pipeline writes both sums; only an empty matrix leaves them to us
    err = torch.empty(2, dtype=torch.float64, device=dev) if rows * n0 else torch.zeros(2, dtype=torch.float64, device=dev)
    padded = -(-rows * n // scale_group) * scale_group
    states = torch.empty((padded // seg, seg), dtype=torch.int32, device=dev) if keep_codes else None
    sc = torch.empty(padded // scale_group, dtype=torch.float32, device=dev) if keep_codes else None
    ws = D.workspace(lib.uq_quant_trellis_workspace_bytes(rows, n0, L, R, seg, scale_group), dev)
    _lib.check(lib.uq_quant_trellis(W.data_ptr(), D.dtype_code(W), rows, n0, n0, H.data_ptr(), L, R, seg,
                                    scale_group, d.data_ptr(), cw.data_ptr(), What.data_ptr(), D.ptr(states),
                                    D.ptr(sc), err.data_ptr(), ws.data_ptr(), ws.numel(), D.stream_handle(dev)),
               "uq_quant_trellis")
    if check_errors:
        _device_status(lib, dev, "uq_quant_trellis")
    return QuantResult(What, err, states, sc)


def quant_step_device(W: torch.Tensor, H: torch.Tensor, step: float, group=256, seed=0,
                      keep_codes=False, block28=False, check_errors=True, scale_search=False) -> QuantResult:
    """Device-resident buildalloc recipe (E8 at a fixed step).  ``block28``
    (opt-in, widths 28 x 512 / 28 x 1024, groups of 256): the unpadded
    block-factorised transform, error sums in the rotated domain.
    ``scale_search`` (opt-in, groups of 256): each row at the best of 16
    steps around ``step`` under the rate constraint of uq_e8_scale_search
    (``choice`` and ``lam`` of the result)."""
    lib = _lib.load()
    dev = W.device
    rows, n0 = W.shape
    if scale_search:
        import ctypes
        if group != 256 or block28:
            raise ValueError("the scale search quantizes groups of 256 of the padded transform")
        n = int(lib.uq_next_pow2(n0))
        H = H.to(device=dev, dtype=torch.float64).contiguous()
        W = W.contiguous()
        d = D.signs(n, seed, dev)
        What = torch.empty((rows, n0), dtype=torch.float32, device=dev)
        err = torch.empty(2, dtype=torch.float64, device=dev) if rows else torch.zeros(2, dtype=torch.float64, device=dev)
        idx = torch.empty(rows * n, dtype=torch.int16, device=dev) if keep_codes else None
        choice = torch.empty(rows, dtype=torch.int32, device=dev)
        lam = ctypes.c_double()
        ws = D.workspace(lib.uq_quant_e8_search_workspace_bytes(rows, n0), dev)
        _lib.check(lib.uq_quant_e8_search(W.data_ptr(), D.dtype_code(W), rows, n0, n0, H.data_ptr(), float(step),
                                          d.data_ptr(), What.data_ptr(), D.ptr(idx), choice.data_ptr(),
                                          ctypes.addressof(lam), err.data_ptr(), ws.data_ptr(), ws.numel(),
                                          D.stream_handle(dev)), "uq_quant_e8_search")
        if check_errors:
            _device_status(lib, dev, "uq_quant_e8_search")
        return QuantResult(What, err, idx=idx, choice=choice, lam=float(lam.value))
    if block28:
        if group != 256:
            raise ValueError("block28 quantizes groups of 256")
        H = H.to(device=dev, dtype=torch.float64).contiguous()
        W = W.contiguous()
        d = D.signs(n0, seed, dev)
        What = torch.empty((rows, n0), dtype=torch.float32, device=dev)
        err = torch.empty(2, dtype=torch.float64, device=dev) if rows else torch.zeros(2, dtype=torch.float64, device=dev)
        idx = torch.empty(rows * n0, dtype=torch.int16, device=dev) if keep_codes else None
        ws = D.workspace(lib.uq_quant_e8_b28_workspace_bytes(rows, n0), dev)
        _lib.check(lib.uq_quant_e8_b28(W.data_ptr(), D.dtype_code(W), rows, n0, n0, H.data_ptr(), float(step),
                                       d.data_ptr(), What.data_ptr(), D.ptr(idx), err.data_ptr(), ws.data_ptr(),
                                       ws.numel(), D.stream_handle(dev)), "uq_quant_e8_b28")
        if check_errors:
            _device_status(lib, dev, "uq_quant_e8_b28")
        return QuantResult(What, err, idx=idx)
    n = int(lib.uq_next_pow2(n0))
    H = H.to(device=dev, dtype=torch.float64).contiguous()
    W = W.contiguous()
    d = D.signs(n, seed, dev)
    What = torch.empty((rows, n0), dtype=torch.float32, device=dev)
    # the pipeline writes both sums; only an empty matrix leaves them to us
    err = torch.empty(2, dtype=torch.float64, device=dev) if rows * n0 else torch.zeros(2, dtype=torch.float64, device=dev)
    idx = torch.empty(-(-rows * n // 8) * 8, dtype=torch.int16, device=dev) if keep_codes else None
    ws = D.workspace(lib.uq_quant_e8_workspace_bytes(rows, n0, group), dev)
    _lib.check(lib.uq_quant_e8(W.data_ptr(), D.dtype_code(W), rows, n0, n0, H.data_ptr(), float(step), group,
                               d.data_ptr(), What.data_ptr(), D.ptr(idx), err.data_ptr(), ws.data_ptr(),
                               ws.numel(), D.stream_handle(dev)), "uq_quant_e8")
    if check_errors:
        _device_status(lib, dev, "uq_quant_e8")
    return QuantResult(What, err, idx=idx)


def _host_result(t: torch.Tensor, like):
    """numpy in -> numpy out; a torch CPU tensor in -> a pinned torch CPU
    tensor out (one device-to-host copy)."""
    if isinstance(like, torch.Tensor):
        out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        out.copy_(t, non_blocking=True)
        torch.cuda.current_stream(t.device).synchronize()
        return out
    return D.to_host(t)


def quant_trellis(W, H, L=12, R=2, seg=64, scale_group=256):
    """buildtrellis.py:16-20 on host arrays: returns What float32 (numpy, or
    a torch CPU tensor when W is one)."""
    w = D.as_device(W)
    h = D.as_device(H, torch.float64)
    return _host_result(quant_trellis_device(w, h, L, R, seg, scale_group, keep_codes=False).What, W)


def quant_step(W, H, step, block28=False, scale_search=False):
    """buildalloc.py:21-24 on host arrays: returns What float32 (``block28``:
    the opt-in unpadded transform for widths 28 x 512 / 28 x 1024;
    ``scale_search``: the opt-in per-row search over 16 steps)."""
    w = D.as_device(W)
    h = D.as_device(H, torch.float64)
    return _host_result(quant_step_device(w, h, step, block28=block28, scale_search=scale_search).What, W)
