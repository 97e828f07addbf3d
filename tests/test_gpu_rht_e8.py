"""GPU parity: RHT / iRHT and the E8 quantizer against the reference goldens
and the oracle (bit-exact), through the C ABI."""
import numpy as np
import pytest

import oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def uq():
    import ultraquant_b200.qlab as Q
    return Q


@pytest.mark.parametrize("tag", list("abcdefghi"))
def test_rht_golden(uq, g_rht, tag):
    A = g_rht[f"rht_{tag}_in"]
    seed = int(g_rht[f"rht_{tag}_seed"])
    X = uq.rht_rows(A, seed=seed)
    assert same_bits(X, g_rht[f"rht_{tag}_out"])
    assert same_bits(uq.irht_rows(X, A.shape[1], seed=seed), g_rht[f"irht_{tag}_out"])
    k = f"irht_{tag}_f32_out"
    if k in g_rht:
        assert same_bits(uq.irht_rows(X.astype(np.float32), A.shape[1], seed=seed), g_rht[k])


@pytest.mark.parametrize("rows,n0", [(1, 2), (3, 17), (7, 255), (5, 256), (9, 4095), (2, 8191), (3, 8192),
                                     (4, 12000), (2, 16384), (33, 64), (3, 16385), (2, 28672), (5, 32768)])
def test_rht_random_vs_oracle(uq, rows, n0):
    rng = np.random.RandomState(rows * 1000 + n0)
    A = rng.standard_t(4, size=(rows, n0)) * 0.02
    X = uq.rht_rows(A)
    assert same_bits(X, O.rht_rows(A))
    assert same_bits(uq.irht_rows(X, n0), O.irht_rows(X, n0))
    X32 = X.astype(np.float32)
    assert same_bits(uq.irht_rows(X32, n0), O.irht_rows(X32, n0))


def test_rht_70b_width(uq):
    """Llama-70B ffn_down width 28672 -> 32768 (row split over a 2-CTA
    cluster): f32 and f64 inputs, forward and inverse, many rows so that every
    cluster walks several rows; bit-exact against the oracle."""
    rng = np.random.RandomState(70)
    A = rng.standard_t(4, size=(300, 28672)) * 0.02
    X = uq.rht_rows(A)
    pick = [0, 1, 149, 298, 299]
    assert same_bits(X[pick], O.rht_rows(A[pick]))
    A32 = A.astype(np.float32)
    assert same_bits(uq.rht_rows(A32)[pick], O.rht_rows(A32[pick]))
    assert same_bits(uq.irht_rows(X, 28672)[pick], O.irht_rows(X[pick], 28672))
    X32 = X.astype(np.float32)
    assert same_bits(uq.irht_rows(X32, 28672)[pick], O.irht_rows(X32[pick], 28672))


def test_pipelines_70b_width():
    """The importance-weighted recipes at the 28672 width (E8 at 0.48 and the
    trellis at L = 12): What bit-exact, weighted NMSE within 1e-5 relative."""
    import torch
    from ultraquant_b200 import pipeline as P
    rng = np.random.RandomState(71)
    W = (rng.standard_t(4, size=(3, 28672)) * 0.015).astype(np.float32)
    H = np.exp(rng.normal(0.0, 1.0, size=28672))
    assert same_bits(P.quant_step(W, H, 0.48), O.quant_step(W.astype(np.float64), H, 0.48))
    res = P.quant_trellis_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), 12, 2, 256, 256)
    ref = O.quant_trellis(W.astype(np.float64), H, L=12, R=2, seg=256)
    assert same_bits(res.What.cpu().numpy(), ref)
    Hc = np.maximum(H, H.max() * 1e-3)
    A = W.astype(np.float64) * np.sqrt(Hc)[None, :]
    Ah = O.irht_rows(O.trellis_quant_fast(O.rht_rows(A), L=12, R=2, seg=256), 28672)
    w = O.wnmse(A, Ah)
    assert abs(res.wnmse - w) <= 1e-5 * w


def test_rht_full_size_roundtrip(uq):
    """4096 x 4096 (and the ffn_down 14336 -> 16384 width): orthogonality and
    a bit-exact subsample of rows against the oracle."""
    import torch
    rng = np.random.RandomState(3)
    for rows, n0 in [(4096, 4096), (1024, 14336)]:
        A = (rng.randn(rows, n0) * 0.02)
        At = torch.from_numpy(A).cuda()
        X = uq.rht_rows(At)
        Ah = uq.irht_rows(X, n0)
        assert float((Ah - At).abs().max()) < 1e-15
        nA, nX = float((At ** 2).sum()), float((X ** 2).sum())
        assert abs(nA - nX) / nA < 1e-12
        pick = rng.choice(rows, 8, replace=False)
        assert same_bits(X[pick].cpu().numpy(), O.rht_rows(A[pick]))


def test_d8_e8_golden(uq, g_e8):
    Y = g_e8["Y"]
    assert same_bits(uq._d8_decode(Y), g_e8["d8"])
    assert same_bits(uq.e8_decode(Y), g_e8["e8"])


def test_e8_random_vs_oracle(uq):
    rng = np.random.RandomState(5)
    Y = np.concatenate([rng.randn(50000, 8) * s for s in (0.3, 1.0, 4.0, 30.0)])
    Y[:1000] = np.round(Y[:1000] * 2) / 2
    assert same_bits(uq.e8_decode(Y), O.e8_decode(Y))
    assert same_bits(uq._d8_decode(Y), O.d8_decode(Y.copy()))


def test_entropy(uq, g_e8):
    v = uq._entropy_bpw(g_e8["ent_pts"])
    ref = float(g_e8["ent_bpw"])
    assert abs(v - ref) <= 1e-12 * ref


def test_q_e8_fixed_golden(uq, g_e8):
    A = g_e8["q_A"]
    for step in (0.48, 0.25, 0.16, 0.11):
        assert same_bits(uq.q_e8_fast(A, fixed_step=step), g_e8[f"q_fixed_{step}"])
    A2 = g_e8["q_A2"]
    assert same_bits(uq.q_e8_fast(A2, fixed_step=0.48), g_e8["q_A2_fixed_0.48"])
    assert same_bits(uq.q_e8_fast(A2, group=64, fixed_step=0.25), g_e8["q_A2_g64_fixed_0.25"])


@pytest.mark.parametrize("group", [8, 64, 128, 256, 512, 1024, 96, 200])
def test_q_e8_groups_vs_oracle(uq, group):
    rng = np.random.RandomState(group)
    A = rng.standard_t(4, size=(37, 301)) * 0.015
    assert same_bits(uq.q_e8_fast(A, group=group, fixed_step=0.48), O.q_e8_fast(A, group=group, fixed_step=0.48))


@pytest.mark.parametrize("tb", [2.0, 3.0])
def test_q_e8_calibrated_golden(uq, g_e8, tb):
    uq._E8_SCALE.clear()
    rec = uq.q_e8_fast(g_e8["q_A3"], target_bpw=tb, calib_key="k")
    assert uq._E8_SCALE["k"] == float(g_e8[f"q_cal_{tb}_step"])
    assert same_bits(rec, g_e8[f"q_cal_{tb}_rec"])
    uq._E8_SCALE.clear()


def test_q_e8_full_size(uq):
    """ffn_down-shaped 4096 x 14336 through rht (pad 16384) and E8 at 0.48:
    rows subsample bit-exact, entropy of the whole index set finite."""
    import torch
    rng = np.random.RandomState(9)
    A = torch.from_numpy(rng.standard_t(4, size=(4096, 14336)) / np.sqrt(2) * 0.015).cuda()
    X = uq.rht_rows(A)
    rec = uq.q_e8_fast(X, fixed_step=0.48)
    pick = [0, 1, 2047, 4095]
    Xs = X[pick].cpu().numpy()
    assert same_bits(rec[pick].cpu().numpy(), O.q_e8_fast(Xs, fixed_step=0.48))
    err = float(((rec - X) ** 2).sum() / (X ** 2).sum())
    assert 0.0 < err < 0.05


@pytest.mark.parametrize("step", [0.48, 0.4, 0.25, 0.11, 1.0 / 3.0])
def test_q_e8_decision_boundaries(uq, step):
    """Inputs whose scaled coordinates sit on or within 1e-12 of rounding
    boundaries (constant-magnitude groups: y = +-c / (|c| + 1e-12) / step),
    exact ties, signed zeros and mixed groups: bit-exact against the oracle
    (the fp32 screen must hand every undecidable vector to the fp64 path)."""
    rng = np.random.RandomState(int(step * 1000))
    groups = []
    for c in (1.0, 1e8, 3.0, 0.5, 1e-3, 7.25):
        for pattern in range(6):
            g = np.full(256, c)
            if pattern == 1:
                g *= rng.choice([-1.0, 1.0], 256)
            elif pattern == 2:
                g[::3] = -c / 2
            elif pattern == 3:
                g[rng.rand(256) < 0.5] = 0.0
            elif pattern == 4:
                g = g * (1 + rng.randint(-3, 4, 256) * 2.0 ** -40)
            elif pattern == 5:
                g = np.round(rng.normal(size=256) * 4) / 2 * c
            groups.append(g)
    groups.append(np.zeros(256))
    groups.append(-np.zeros(256))
    z = np.zeros(256)
    z[::2] = -0.0
    z[1::2] = 1e-300
    groups.append(z)
    A = np.concatenate(groups).reshape(-1, 256)
    got = uq.q_e8_fast(A, fixed_step=step)
    ref = O.q_e8_fast(A, fixed_step=step)
    assert same_bits(got, ref)


def test_q_e8_many_rows_vs_oracle(uq):
    """1 M elements of Student-t data (131 K vectors, a few hundred of them
    decided by the exact fp64 path): bit-exact."""
    rng = np.random.RandomState(21)
    A = rng.standard_t(4, size=(64, 16384)) * 0.02
    for step in (0.48, 0.3):
        assert same_bits(uq.q_e8_fast(A, fixed_step=step), O.q_e8_fast(A, fixed_step=step))


def test_wnmse_vs_oracle(uq):
    """qlab.wnmse on the device: fp64 sums, within 1e-12 relative of numpy's."""
    rng = np.random.RandomState(5)
    A = rng.normal(size=(300, 1000))
    Ah = A + 0.01 * rng.normal(size=A.shape)
    for a, b in ((A, Ah), (A.astype(np.float32), Ah), (A, Ah.astype(np.float32))):
        ref = O.wnmse(np.asarray(a, np.float64), np.asarray(b, np.float64))
        assert abs(uq.wnmse(a, b) - ref) <= 1e-12 * ref
    assert uq.wnmse(A, A) == 0.0


@pytest.mark.parametrize("rows,n0", [(1, 14336), (3, 28672), (150, 14336)])
def test_block28_vs_oracle(uq, rows, n0):
    """Opt-in unpadded 28 x P transform (no reference counterpart): forward
    and inverse bit-exact against the oracle's operation order, f32 / f64 input."""
    rng = np.random.RandomState(rows + n0)
    A = rng.standard_t(4, size=(rows, n0)) * 0.02
    pick = sorted({0, rows // 2, rows - 1})
    X = uq.rht_rows(A, block28=True)
    assert same_bits(X[pick], O.rht28_rows(A[pick]))
    A32 = A.astype(np.float32)
    assert same_bits(uq.rht_rows(A32, block28=True)[pick], O.rht28_rows(A32[pick]))
    assert same_bits(uq.irht_rows(X, n0, block28=True)[pick], O.irht28_rows(X[pick]))


def test_quant_step_block28_vs_oracle():
    """Opt-in buildalloc recipe on an ffn_down-shaped slice with the unpadded
    transform: What bit-exact, weighted NMSE (rotated domain) within 1e-12 of
    the oracle's and within 1e-6 of the original-domain value."""
    import torch
    from ultraquant_b200 import pipeline as P
    rng = np.random.RandomState(29)
    W = (rng.standard_t(4, size=(8, 14336)) / np.sqrt(2) * 0.015).astype(np.float32)
    H = np.exp(rng.normal(0.0, 1.0, size=14336))
    res = P.quant_step_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), 0.48, block28=True)
    ref, X, Xq = O.quant_step_b28(W.astype(np.float64), H, 0.48)
    assert same_bits(res.What.cpu().numpy(), ref)
    w_rot = float(np.sum((X - Xq) ** 2) / np.sum(X ** 2))
    assert abs(res.wnmse - w_rot) <= 1e-12 * w_rot
    Hc = np.maximum(H, H.max() * 1e-3)
    A = W.astype(np.float64) * np.sqrt(Hc)[None, :]
    Ah = ref.astype(np.float64) * np.sqrt(Hc)[None, :]
    assert abs(res.wnmse - O.wnmse(A, Ah)) <= 1e-6 * res.wnmse + 1e-6


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_q_uniform_golden(uq, g_quniform, tag):
    """qlab.q_uniform (lab quantizer): bit-exact against the reference in both dtypes."""
    A = g_quniform[f"qu_{tag}_A"]
    for bpw in (2, 3, 4, 2.5):
        got = uq.q_uniform(A, bpw)
        assert got.dtype == A.dtype and same_bits(got, g_quniform[f"qu_{tag}_{bpw}"])
    assert same_bits(uq.q_uniform(A, 3, bs=64), g_quniform[f"qu_{tag}_bs64"])
    rng = np.random.RandomState(3)
    B = rng.normal(size=(64, 4096))
    assert same_bits(uq.q_uniform(B, 3), O.q_uniform(B, 3))
    with pytest.raises(ValueError):
        uq.q_uniform(np.zeros((3, 10)), 2)


def test_sharded_e8_calibration_device(uq):
    """The calibration pieces of a row-sharded tensor (sample ids, device gn
    of the local vectors, device bisection) give the single-call step, with
    the tensor held as three uneven row blocks by one process."""
    import torch
    from ultraquant_b200 import shard as S
    rng = np.random.RandomState(12)
    W = rng.standard_t(4, size=(300, 1024)) * 0.02
    uq._E8_SCALE.pop("shard", None)
    whole = uq.q_e8_fast(W, target_bpw=2.5, calib_key="shard")
    step_whole = uq._E8_SCALE.pop("shard")
    cache = {}
    O.q_e8_fast(W, 2.5, calib_key="o", cache=cache)
    assert step_whole == cache["o"]
    spec = S.TensorSpec("w", 300, 1024)
    cuts = [0, 7, 160, 300]
    blocks = [(cuts[i], torch.from_numpy(W[cuts[i]:cuts[i + 1]]).cuda()) for i in range(3)]
    assert S.calibrate_e8(blocks, spec, 2.5) == step_whole
    assert whole.shape == W.shape
