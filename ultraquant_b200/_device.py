"""Device plumbing for the Python layer: CUDA tensors, streams and caches.

PyTorch provides device memory, host<->device copies and the current stream;
all arithmetic happens in libuq_b200.  Host numpy arrays given to the
reference-compatible functions are copied in and the results copied back,
exactly like the reference's own ``torch.tensor(..., device)`` /
``.cpu().numpy()`` boundary.
"""
from __future__ import annotations

import threading

import numpy as np
import torch

from . import _lib
from ._lib import UQ_F32, UQ_F64

_tls = threading.local()
_cache_lock = threading.Lock()
_signs_cache: dict = {}
_codebook_cache: dict = {}


def device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("ultraquant_b200 needs a CUDA device (sm_100a); none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def stream_handle(dev: torch.device | None = None) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return UQ_F32
    if t.dtype == torch.float64:
        return UQ_F64
    raise TypeError(f"unsupported dtype {t.dtype} (float32 / float64 expected)")


def as_device(a, dtype=None, dev: torch.device | None = None) -> torch.Tensor:
    """numpy / torch input -> contiguous CUDA tensor (float32 or float64)."""
    dev = dev or device()
    if isinstance(a, torch.Tensor):
        t = a
    else:
        arr = np.asarray(a)
        if dtype is None and arr.dtype not in (np.float32, np.float64):
            arr = arr.astype(np.float64)
        t = torch.from_numpy(np.ascontiguousarray(arr))
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if t.dtype not in (torch.float32, torch.float64, torch.int32, torch.int64, torch.int16):
        t = t.to(torch.float64)
    if t.device != dev:
        if t.device.type == "cpu" and not t.is_pinned() and t.numel() * t.element_size() >= (1 << 20):
            t = t.pin_memory()
        t = t.to(dev, non_blocking=True)
    return t.contiguous()


def workspace(nbytes: int, dev: torch.device | None = None) -> torch.Tensor:
    """A per-thread, per-device growing scratch buffer (uint8)."""
    dev = dev or device()
    key = ("ws", dev.index)
    cur = getattr(_tls, "ws", {}).get(key)
    if cur is None or cur.numel() < nbytes:
        cur = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
        if not hasattr(_tls, "ws"):
            _tls.ws = {}
        _tls.ws[key] = cur
    return cur


def signs(n: int, seed: int = 0, dev: torch.device | None = None) -> torch.Tensor:
    """Device copy of the RHT sign vector (MT19937 on the host, cached)."""
    dev = dev or device()
    key = (dev.index, int(seed), int(n))
    with _cache_lock:
        t = _signs_cache.get(key)
    if t is None:
        lib = _lib.load()
        host = np.empty(n, np.float64)
        _lib.check(lib.uq_rht_signs(int(seed) & 0xFFFFFFFF, n, host.ctypes.data), "uq_rht_signs")
        t = torch.from_numpy(host).to(dev)
        with _cache_lock:
            _signs_cache[key] = t
    return t


def codebook(L: int, dev: torch.device | None = None) -> torch.Tensor:
    """Device codebook for L state bits (AS241 kernel; prefixes of L=16)."""
    dev = dev or device()
    key = (dev.index, int(L))
    with _cache_lock:
        t = _codebook_cache.get(key)
    if t is None:
        lib = _lib.load()
        t = torch.empty(1 << L, dtype=torch.float32, device=dev)
        _lib.check(lib.uq_trellis_codebook(int(L), t.data_ptr(), stream_handle(dev)), "uq_trellis_codebook")
        with _cache_lock:
            _codebook_cache[key] = t
    return t


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()
