"""ctypes binding of ``libuq_b200.so`` (declared in ``include/uq_b200.h``).

The library is the product: there is no CPU fallback.  If it is missing or
no CUDA device is visible, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libuq_b200.so")

UQ_OK, UQ_ERR_INVALID, UQ_ERR_UNSUPPORTED, UQ_ERR_CUDA, UQ_ERR_WORKSPACE, UQ_ERR_TIMEOUT = range(6)
UQ_F32, UQ_F64 = 0, 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_u32 = ctypes.c_uint32
_f64 = ctypes.c_double
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/uq_b200.h
SIGNATURES = {
    "uq_version": (_i32, []),
    "uq_status_string": (ctypes.c_char_p, [_i32]),
    "uq_last_error": (ctypes.c_char_p, []),
    "uq_next_pow2": (_i64, [_i64]),
    "uq_rht_signs": (_i32, [_u32, _i64, _p]),
    "uq_rht_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p]),
    "uq_irht_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "uq_rht28_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p]),
    "uq_irht28_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i32, _i64, _p]),
    "uq_q_uniform": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p]),
    "uq_q_e8_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_q_e8": (_i32, [_p, _i32, _i64, _i64, _p, _p, _i64, _f64, _f64, _p, _p, _sz, _p]),
    "uq_d8_decode": (_i32, [_p, _i64, _p, _p]),
    "uq_e8_decode": (_i32, [_p, _i64, _p, _p]),
    "uq_e8_quant": (_i32, [_p, _i32, _i64, _i64, _f64, _p, _p, _p]),
    "uq_e8_entropy_workspace_bytes": (_sz, [_i64]),
    "uq_e8_entropy_bpw": (_i32, [_p, _i64, _p, _p, _sz, _p]),
    "uq_e8_calibrate_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_e8_calibrate": (_i32, [_p, _i32, _i64, _i64, _f64, _p, _p, _sz, _p]),
    "uq_e8_sample_indices": (_i32, [_i64, _i64, _p]),
    "uq_e8_sample_gn_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_e8_sample_gn": (_i32, [_p, _i32, _i64, _i64, _p, _i64, _p, _p, _sz, _p]),
    "uq_e8_calibrate_sample_workspace_bytes": (_sz, [_i64]),
    "uq_e8_calibrate_sample": (_i32, [_p, _i64, _f64, _p, _p, _sz, _p]),
    "uq_e8_scale_search_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_e8_scale_search": (_i32, [_p, _i64, _i64, _f64, _p, _p, _p, _p, _p, _sz, _p]),
    "uq_quant_e8_search_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_quant_e8_search": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _f64, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "uq_trellis_codebook": (_i32, [_i32, _p, _p]),
    "uq_trellis_normalize": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p]),
    "uq_trellis_normalize_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "uq_trellis_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32]),
    "uq_trellis_viterbi": (_i32, [_p, _i64, _i32, _i32, _i32, _p, _p, _p, _sz, _p]),
    "uq_trellis_noalloc_scratch_bytes": (_sz, []),
    "uq_trellis_viterbi_noalloc": (_i32, [_p, _i64, _i32, _i32, _i32, _p, _p, _p]),
    "uq_trellis_decode": (_i32, [_p, _p, _p, _i64, _i64, _p, _p]),
    "uq_trellis_decode_rows": (_i32, [_p, _p, _p, _i64, _i64, _i64, _i64, _p, _p]),
    "uq_trellis_packed_words": (_i64, [_i32, _i32, _i32]),
    "uq_trellis_pack": (_i32, [_p, _i64, _i32, _i32, _i32, _p, _p]),
    "uq_trellis_unpack": (_i32, [_p, _i64, _i32, _i32, _i32, _p, _p]),
    "uq_wnmse_workspace_bytes": (_sz, []),
    "uq_wnmse_sums": (_i32, [_p, _i32, _p, _i32, _i64, _p, _p, _sz, _p]),
    "uq_q8_encode": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p]),
    "uq_q8_decode": (_i32, [_p, _i64, _i64, _p, _i64, _p]),
    "uq_fwht": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _p, _p, _i32, _p, _i64, _i64, _p]),
    "uq_qat_recon": (_i32, [_p, _i32, _i64, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _p]),
    "uq_qat_recon_backward_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_qat_recon_backward": (_i32, [_p, _i64, _p, _i32, _i64, _i64, _p, _i64, _p, _i64, _i64, _p, _p,
                                     _i64, _p, _p, _p, _sz, _p]),
    "uq_quant_trellis_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32, _i32, _i32]),
    "uq_quant_trellis": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _p, _p, _p, _p,
                                _p, _p, _p, _sz, _p]),
    "uq_quant_e8_workspace_bytes": (_sz, [_i64, _i64, _i32]),
    "uq_quant_e8": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _f64, _i32, _p, _p, _p, _p, _p, _sz, _p]),
    "uq_quant_e8_b28_workspace_bytes": (_sz, [_i64, _i64]),
    "uq_quant_e8_b28": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _f64, _p, _p, _p, _p, _p, _sz, _p]),
    "uq_device_errors": (_i32, [_p]),
    "uq_wait_timeout_selftest": (_i32, [_f64, _p]),
    "uq_inject_device_flag": (_i32, [_i32]),
    "uq_profile_enable": (None, [_i32]),
    "uq_profile_reset": (None, []),
    "uq_launch_count": (_i64, []),
    "uq_profile_read": (_i32, [ctypes.c_char_p, _p, _p]),
    "uq_fp32_lane_probe": (_i32, [_i32, _i64, _p, _p]),
}

_lock = threading.Lock()
_lib = None


class UQError(RuntimeError):
    """A CUDA-side failure reported by libuq_b200 (status UQ_ERR_CUDA / TIMEOUT)."""


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once and attach prototypes.  Raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m ultraquant_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    """Map a uq_status to the exception the reference would raise."""
    if rc == UQ_OK:
        return
    lib = load()
    msg = f"{what}: {lib.uq_last_error().decode(errors='replace')}"
    if rc == UQ_ERR_INVALID:
        raise ValueError(msg)
    if rc == UQ_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == UQ_ERR_WORKSPACE:
        raise MemoryError(msg)
    raise UQError(msg)
