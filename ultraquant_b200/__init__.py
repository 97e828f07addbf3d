"""ultraquant_b200 -- UltraQuant's weight-quantization hot path on B200 (sm_100a).

Modules mirror the reference's interfaces:

* ``ultraquant_b200.qlab``     -- rht_rows, irht_rows, e8_decode, q_e8_fast, ...
* ``ultraquant_b200.trellis``  -- codebook, trellis_quant, trellis_quant_fast
* ``ultraquant_b200.qat``      -- trellis_encode, fwht_torch, irht_torch, recon_torch
* ``ultraquant_b200.q8``       -- enc_q8 / deq_q8 (Q8_0 blocks of the GGUF container)
* ``ultraquant_b200.pipeline`` -- the builders' importance-weighted recipes
* ``ultraquant_b200.shard``    -- row-block sharding over torch.distributed ranks

All arithmetic runs in ``libuq_b200.so`` (C ABI in ``include/uq_b200.h``).
``install()`` swaps these functions into already-importable reference modules
so that unmodified builders (buildtrellis.py, buildalloc.py, qat.py) run on
the GPU path.
"""
from __future__ import annotations

import importlib
import sys

from ._lib import LIB_PATH, load  # noqa: F401

__version__ = "0.1.0"

_PATCH = {
    "qlab": ("_next_pow2", "rht_rows", "irht_rows", "_d8_decode", "e8_decode", "_entropy_bpw",
             "q_e8_fast", "wnmse", "deq_q8", "q_uniform", "e8_codebook", "q_e8"),
    "trellis": ("codebook", "pred_table", "trellis_quant", "trellis_quant_fast"),
    "qat": ("trellis_encode", "fwht_torch", "irht_torch", "recon_torch"),
    "buildq": ("enc_q8",),
}
_SOURCE = {"buildq": "q8"}   # reference module -> module of this package


def install(modules=("qlab", "trellis", "qat")):
    """Replace the hot-path functions of the reference modules ``qlab``,
    ``trellis`` and ``qat`` (imported from ``sys.path``) by this package's;
    add ``"buildq"`` to also replace its ``enc_q8``.
    Call it before the builders run ``from qlab import rht_rows``.  Returns
    the patched module objects."""
    patched = {}
    for name in modules:
        ref = importlib.import_module(name)
        mine = importlib.import_module(f"{__name__}.{_SOURCE.get(name, name)}")
        for attr in _PATCH[name]:
            setattr(ref, attr, getattr(mine, attr))
        if name == "qlab":
            ref._E8_SCALE = mine._E8_SCALE
        patched[name] = ref
        sys.modules[name] = ref
    return patched
