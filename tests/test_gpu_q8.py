"""GPU parity of the Q8_0 block codec (buildq.py:21-30 enc_q8, qlab.py:27-32
deq_q8): bytes and values bit-exact against the reference goldens and the
oracle, through the C ABI."""
import numpy as np
import pytest

import oracle as O
from conftest import same_bits, same_bits_or_nan

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Q8():
    import ultraquant_b200.q8 as Q8
    return Q8


@pytest.mark.parametrize("tag", ["f32", "f64"])
def test_q8_golden(Q8, g_q8, tag):
    W = g_q8[f"q8_{tag}_W"]
    q = Q8.enc_q8(W)
    assert q.dtype == np.uint8 and np.array_equal(q, g_q8[f"q8_{tag}_enc"])

    class T:
        data = g_q8[f"q8_{tag}_enc"]
    assert same_bits(Q8.deq_q8(T()), g_q8[f"q8_{tag}_dec"])


@pytest.mark.parametrize("rows,cols", [(1, 32), (3, 96), (7, 1056), (64, 4096), (5, 32 * 33)])
def test_q8_random_vs_oracle(Q8, rows, cols):
    rng = np.random.RandomState(rows + cols)
    W = (rng.standard_t(3, size=(rows, cols)) * 0.03).astype(np.float32)
    W[:, :32] *= rng.choice([0.0, 1.0, 1e5], size=(rows, 1))
    q = Q8.enc_q8(W)
    assert np.array_equal(q, O.enc_q8(W))
    assert same_bits(Q8.deq_q8(q), O.deq_q8(q))


def test_q8_device_tensors_and_errors(Q8):
    import torch
    W = torch.randn(128, 4096, device="cuda") * 0.02
    q = Q8.enc_q8(W)
    assert q.is_cuda and q.shape == (128, 128 * 34)
    back = Q8.deq_q8(q)
    assert back.is_cuda and back.shape == (128, 4096)
    ref = O.deq_q8(O.enc_q8(W.cpu().numpy()))
    assert same_bits(back.cpu().numpy(), ref)
    with pytest.raises(ValueError):
        Q8.enc_q8(np.zeros((2, 33), np.float32))


def test_q8_rounding_ties_and_extreme_scales(Q8):
    """Values on the rounding boundaries (x / scale = k + 1/2 exactly, where
    the reciprocal screen must hand over to the division) and scales at the
    ends of the fp32 range (the scale's own division fallback, subnormal
    scales whose reciprocal overflows), against the oracle."""
    rng = np.random.RandomState(7)
    rows = []
    for e in (-140, -126, -101, -100, -30, 0, 30, 99, 100, 101):
        s = np.float32(2.0 ** e)
        k = rng.randint(-126, 126, size=31)
        blk = np.concatenate([[127.0], k + 0.5]) * np.float64(s)
        rows.append(rng.permutation(blk))
        # the same values scaled by a non-power of two (scale no longer exact)
        rows.append(rng.permutation(blk) * 1.37)
    W = np.asarray(rows, dtype=np.float32).reshape(len(rows), 32)
    W = np.concatenate([W, np.zeros((1, 32), np.float32), -W[:3]], axis=0)
    with np.errstate(over="ignore"):   # float16 scales of 2^100 and up are inf
        ref = O.enc_q8(W)
    q = Q8.enc_q8(W)
    assert np.array_equal(q, ref)
    # an inf scale times q = 0 is NaN
    with np.errstate(invalid="ignore"):
        assert same_bits_or_nan(Q8.deq_q8(q), O.deq_q8(q))
