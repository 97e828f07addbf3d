"""L = 16 parity on the benchmarked tensor and on Llama-3.1-8B tensor shapes.

The device recipe (buildtrellis.py:16-20 around trellis.py:62-108: clamp the
imatrix, A = W*sqrt(H), RHT, per-256 RMS, Viterbi with L = 16 and T = 256,
decode, inverse RHT, /sqrt(H)) runs on the WHOLE tensor; the oracle
recomputes a spread sample of rows (RHT, normalisation and trellis segments
never cross rows, because every padded width is a multiple of 256) and the
test compares, per sampled row:

* the per-256 scales and the trellis state paths (bit-exact; a differing
  path is accepted only as an exact fp32 cost tie, and at most 0.01 % of the
  sequences may differ at all);
* the reconstruction What (bit-exact);
* the weighted reconstruction error of the sampled rows, run as a tensor of
  its own, within 1e-5 relative.

The oracle's Viterbi is the C restatement (oracle/uq_viterbi_ref.c), pinned
against the reference goldens on the CPU.  ``UQ_PARITY_FULL=1`` checks every
row instead of the sample (minutes of host time).
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import same_bits
from oracle import cviterbi as CV
from oracle.uq_oracle import _flat_normalise

pytestmark = pytest.mark.gpu

FULL = os.environ.get("UQ_PARITY_FULL", "") == "1"


def _student_t(rng, shape, std):
    # Student-t with nu = 4 has variance 2: scale to the given std
    return (rng.standard_t(4, size=shape) / np.sqrt(2.0) * std).astype(np.float32)


def _oracle_rows(W, H, rows, L, R, seg=256, group=256):
    """Oracle recipe on the given rows: (xn, sc, states, Ah fp64, A fp64, What)."""
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = W[rows].astype(np.float64) * sH
    n0 = A.shape[1]
    Ar = O.rht_rows(A)
    xn, sc_g, ntot, _ = _flat_normalise(Ar, seg, group)
    cw = O.codebook(L)
    st = CV.viterbi_segments_c(xn, L, R, cw)
    meta = dict(scale_group=group, Ntot=ntot, nrow=Ar.shape[0], ncol=Ar.shape[1])
    Ah = O.irht_rows(O.trellis_decode(st.astype(np.int32), cw, sc_g, meta), n0)
    return xn, sc_g.reshape(-1), st, Ah, A, (Ah / sH).astype(np.float32)


def _check_tensor(W, H, R, nsample_rows, seed, L=16, seg=256, group=256):
    import torch
    from ultraquant_b200 import pipeline as P
    rows_n, n0 = W.shape
    n = O.next_pow2(n0)
    spr = n // seg                      # sequences per row
    gpr = n // group                    # scale groups per row
    res = P.quant_trellis_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), L, R, seg, group)
    st_dev = res.states.cpu().numpy()
    sc_dev = res.sc.cpu().numpy()
    What_dev = res.What.cpu().numpy()
    assert st_dev.shape == (rows_n * spr, seg)
    if FULL or nsample_rows >= rows_n:
        rows = np.arange(rows_n)
    else:
        rng = np.random.RandomState(seed)
        rows = np.sort(rng.choice(rows_n, nsample_rows, replace=False))
    mism = 0
    nseq = 0
    for b0 in range(0, rows.size, 512):
        blk = rows[b0:b0 + 512]
        xn, sc, st, _, _, What = _oracle_rows(W, H, blk, L, R, seg, group)
        sidx = (blk[:, None] * spr + np.arange(spr)[None, :]).ravel()
        gidx = (blk[:, None] * gpr + np.arange(gpr)[None, :]).ravel()
        assert same_bits(sc_dev[gidx], sc), "per-256 scales differ"
        got = st_dev[sidx].astype(np.int64)
        bad = np.flatnonzero((got != st).any(1))
        nseq += sidx.size
        if bad.size:
            # every differing path must be an exact fp32 cost tie
            cg = CV.path_costs(xn[bad], got[bad], L)
            co = CV.path_costs(xn[bad], st[bad], L)
            assert np.array_equal(cg.view(np.int32), co.view(np.int32)), \
                f"{bad.size} sequences differ and are not cost ties"
            mism += bad.size
        # What is bit-exact on every row whose paths all match
        ok = np.ones(blk.size, bool)
        ok[np.unique(bad // spr)] = False
        assert same_bits(What_dev[blk[ok]], What[ok]), "What differs"
    assert mism <= 1e-4 * nseq, f"{mism} of {nseq} sequences differ (bar: 99.99 % identical)"
    # weighted error of a slice of the sampled rows, run as a tensor of its own
    sub = rows[:64]
    r2 = P.quant_trellis_device(torch.from_numpy(np.ascontiguousarray(W[sub])).cuda(), torch.from_numpy(H).cuda(),
                                L, R, seg, group, keep_codes=False)
    _, _, _, Ah, A, _ = _oracle_rows(W, H, sub, L, R, seg, group)
    ref = O.wnmse(A, Ah)
    assert abs(r2.wnmse - ref) <= 1e-5 * ref, (r2.wnmse, ref)
    return nseq, mism, res.wnmse


@pytest.mark.parametrize("R", [2, 3])
def test_bench_tensor_l16(R):
    """The benchmarked 4096 x 4096 tensor (N(0, 0.02^2), 0.1 % of entries at
    +-8 sigma, log-normal imatrix; seed 0) at L = 16, T = 256: 8,192 of the
    65,536 sequences (512 rows spread over the tensor)."""
    import bench
    W, H = bench.make_inputs(0)
    nseq, mism, w = _check_tensor(W, H, R, 512, seed=100 + R)
    assert nseq >= 8192 or FULL
    assert 0.0 < w < (0.08 if R == 2 else 0.03)


@pytest.mark.parametrize("name,rows,cols,R", [
    ("ffn_down", 4096, 14336, 3),       # padded to 16384 columns: 64 sequences per row
    ("ffn_gate", 14336, 4096, 2),
    ("attn_k", 1024, 4096, 2),
])
def test_llama8b_shapes_l16(name, rows, cols, R):
    """Llama-3.1-8B tensor shapes with Student-t (nu = 4) weights of std 0.02
    and a log-normal imatrix, at the k of the searched allocation: 4,096
    sequences per tensor checked."""
    rng = np.random.RandomState(sum(map(ord, name)))
    W = _student_t(rng, (rows, cols), 0.02)
    H = np.exp(rng.normal(0.0, 1.0, size=cols))
    spr = O.next_pow2(cols) // 256
    nseq, mism, w = _check_tensor(W, H, R, 4096 // spr, seed=7)
    assert nseq >= 4096


@pytest.mark.parametrize("name,rows,cols", [
    ("ffn_down", 8192, 28672),          # padded to 32768 columns (2-CTA transform): 128 sequences per row
    ("ffn_gate", 28672, 8192),
    ("attn_k", 1024, 8192),
])
def test_llama70b_shapes_l16(name, rows, cols):
    """Llama-3-70B tensor shapes with Student-t (nu = 4) weights of std 0.015
    and a log-normal imatrix at the uniform k = 2 of that weight set: 4,096
    sequences per tensor checked."""
    rng = np.random.RandomState(sum(map(ord, name)) + 70)
    W = _student_t(rng, (rows, cols), 0.015)
    H = np.exp(rng.normal(0.0, 1.0, size=cols))
    spr = O.next_pow2(cols) // 256
    nseq, mism, w = _check_tensor(W, H, 2, 4096 // spr, seed=70)
    assert nseq >= 4096
    assert 0.0 < w < 0.08
