"""Drop-in replacements for the Q8_0 block codec of UltraQuant's builders:
``enc_q8`` (buildq.py:21-30) and ``deq_q8`` (qlab.py:27-32).

Bytes and values equal the reference's; numpy in -> numpy out, CUDA tensors
in -> CUDA tensors out.  ``deq_q8`` accepts a GGUF tensor object (anything
with ``.data``) like the reference, or the raw (rows, blocks * 34) bytes.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _device as D
from . import _lib

__all__ = ["enc_q8", "deq_q8"]


def enc_q8(W):
    """buildq.py:21-30 -- (rows, cols) -> (rows, cols // 32 * 34) uint8."""
    lib = _lib.load()
    on_dev = isinstance(W, torch.Tensor) and W.is_cuda
    w = D.as_device(W)
    if w.dim() != 2:
        raise ValueError(f"enc_q8: expected a 2-D matrix, got shape {tuple(w.shape)}")
    rows, cols = w.shape
    if cols % 32:
        raise ValueError(f"cannot reshape array of size {rows * cols} into shape ({rows},{cols // 32},32)")
    out = torch.empty((rows, cols // 32 * 34), dtype=torch.uint8, device=w.device)
    _lib.check(lib.uq_q8_encode(w.data_ptr() if w.numel() else None, D.dtype_code(w), rows, cols, max(cols, 1),
                                out.data_ptr() if out.numel() else None, D.stream_handle(w.device)), "enc_q8")
    return out if on_dev else D.to_host(out)


def deq_q8(t):
    """qlab.py:27-32 -- Q8_0 rows (rows, blocks * 34) -> (rows, blocks * 32) float32."""
    lib = _lib.load()
    data = getattr(t, "data", t)
    on_dev = isinstance(data, torch.Tensor) and data.is_cuda
    if isinstance(data, torch.Tensor):
        q = data.to(torch.uint8)
    else:
        q = torch.from_numpy(np.ascontiguousarray(np.asarray(data, dtype=np.uint8)))
    q = q.to(D.device() if not on_dev else q.device).contiguous()
    rows, brow = q.shape
    nb = brow // 34
    if brow != nb * 34:
        raise ValueError(f"cannot reshape array of size {rows * brow} into shape ({rows},{nb},34)")
    out = torch.empty((rows, nb * 32), dtype=torch.float32, device=q.device)
    _lib.check(lib.uq_q8_decode(q.data_ptr() if q.numel() else None, rows, nb * 32,
                                out.data_ptr() if out.numel() else None, max(nb * 32, 1),
                                D.stream_handle(q.device)), "deq_q8")
    return out if on_dev else D.to_host(out)
