"""Drop-in replacement for the encoder of UltraQuant's ``qat.py`` (qat.py:11-33).

``trellis_encode`` returns the reference's tuple
``(states (Nseg, seg) int32, sc_g (G, 1) float32, cw (2^L,) float32, meta)``.
"""
from __future__ import annotations

import numpy as np

from . import _device as D
from .trellis import encode_segments

__all__ = ["DEV", "trellis_encode"]

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
