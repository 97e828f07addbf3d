"""The opt-in per-row scale search of the E8 quantizer (config 3's 16
candidate scales; no counterpart in the reference, so its parity is defined
by the oracle's restatement, oracle/uq_oracle.py e8_scale_search): the
device search returns the oracle's choice per row, lam and reconstruction
bit for bit, alone and inside the buildalloc recipe."""
import numpy as np
import pytest

import oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n,step,seed", [(64, 2048, 0.48, 0), (40, 4096, 0.25, 1), (8, 256, 0.48, 2),
                                              (16, 16384, 0.48, 3), (3, 512, 1.0, 4)])
def test_scale_search_matches_oracle(rows, n, step, seed):
    from ultraquant_b200 import qlab as Q
    rng = np.random.RandomState(seed)
    A = O.rht_rows(rng.standard_t(4, size=(rows, n)) / np.sqrt(2) * 0.015)
    rec, choice, lam = Q.e8_scale_search(A, step)
    ref, rchoice, rlam = O.e8_scale_search(A, step)
    assert np.array_equal(choice, rchoice.astype(np.int32))
    assert lam == rlam
    assert same_bits(rec, ref)


def test_scale_search_edge_rows():
    """Rows of zeros (every candidate costs nothing), a row with one large
    outlier and rows at very different scales."""
    from ultraquant_b200 import qlab as Q
    rng = np.random.RandomState(7)
    A = rng.normal(0, 1, size=(6, 1024))
    A[0] = 0.0
    A[1, 17] = 40.0
    A[2] *= 1e-6
    A[3] *= 1e3
    rec, choice, lam = Q.e8_scale_search(A, 0.48)
    ref, rchoice, rlam = O.e8_scale_search(A, 0.48)
    assert np.array_equal(choice, rchoice.astype(np.int32)) and lam == rlam
    assert same_bits(rec, ref)


def test_quant_step_scale_search_recipe():
    """buildalloc.py:21-24 with the search in place of the fixed step:
    What bit-exact with the oracle's composition, weighted NMSE within
    1e-5 (and close to the fixed step's: the search trades error against a
    rate no higher than the fixed step's, so it can land on either side)."""
    import torch
    from ultraquant_b200 import pipeline as P
    rng = np.random.RandomState(5)
    W = (rng.standard_t(4, size=(48, 1500)) / np.sqrt(2) * 0.015)
    H = np.exp(rng.normal(0, 1, size=1500))
    res = P.quant_step_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), 0.48, scale_search=True)
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = W * sH
    rec, choice, lam = O.e8_scale_search(O.rht_rows(A), 0.48)
    Ah = O.irht_rows(rec, W.shape[1])
    assert np.array_equal(res.choice.cpu().numpy(), choice.astype(np.int32)) and res.lam == lam
    assert same_bits(res.What.cpu().numpy(), (Ah / sH).astype(np.float32))
    ref = O.wnmse(A, Ah)
    assert abs(res.wnmse - ref) <= 1e-5 * ref
    fixed = P.quant_step_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), 0.48)
    assert abs(res.wnmse - fixed.wnmse) <= 0.05 * fixed.wnmse


def test_scale_search_rejects_bad_shapes():
    from ultraquant_b200 import qlab as Q
    with pytest.raises(ValueError):
        Q.e8_scale_search(np.zeros((4, 300)), 0.48)       # not a multiple of 256
    with pytest.raises(ValueError):
        Q.e8_scale_search(np.zeros((4, 512)), 0.0)
