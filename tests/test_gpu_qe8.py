"""GPU parity: the finite-codebook E8 quantizer (qlab.q_e8, qlab.py:185-198)
against the reference goldens, the oracle and a torch fp64 brute force."""
import numpy as np
import pytest

import oracle as O
from conftest import qe8_same_or_tie, same_bits
from test_oracle_golden import QE8_CASES, _qe8_input

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def uq():
    import ultraquant_b200.qlab as Q
    return Q


@pytest.mark.parametrize("case", QE8_CASES, ids=[c[1] for c in QE8_CASES])
def test_q_e8_golden(uq, g_qe8, case):
    key, out, bpw, group, f32 = case
    A = _qe8_input(g_qe8, key, f32)
    got = uq.q_e8(A, bpw, group)
    assert got.dtype == np.float64
    # bit-exact but for exact distance ties, which cKDTree breaks by its search order
    assert qe8_same_or_tie(got, g_qe8[out], A, bpw, group) >= 0
    assert same_bits(got, O.q_e8(A, bpw, group))


def test_q_e8_golden_group64(uq, g_qe8):
    A = g_qe8["qe_A"][:8]
    assert same_bits(uq.q_e8(A, 2.0, group_scale=64), g_qe8["qe_A_g64_2.0"])


@pytest.mark.parametrize("shape,bpw,group", [((24, 512), 2.0, 256), ((3, 4096), 1.5, 128), ((5, 96), 1.0, 32),
                                             ((2, 3), 2.0, 8), ((4, 1000), 2.0, 256)])
def test_q_e8_vs_oracle(uq, shape, bpw, group):
    rng = np.random.RandomState(shape[0] * 7 + shape[1])
    A = rng.standard_t(4, size=shape) * 0.02
    assert same_bits(uq.q_e8(A, bpw, group), O.q_e8(A, bpw, group))


def _search_only(uq, A, bpw, group=256):
    """q_e8 through the C ABI with the lattice shortcut disabled (norm_cut 0):
    every vector goes through the codebook search."""
    import torch
    from ultraquant_b200 import _device as D, _lib
    lib = _lib.load()
    a = D.as_device(A)
    cb, cb32, scale, _ = uq._e8_codebook_dev(1 << int(round(bpw * 8)), a.device)
    out = torch.empty(a.shape, dtype=torch.float64, device=a.device)
    ws = D.workspace(lib.uq_q_e8_workspace_bytes(a.numel(), group), a.device)
    _lib.check(lib.uq_q_e8(a.data_ptr(), D.dtype_code(a), a.numel(), group, cb.data_ptr(), cb32.data_ptr(),
                           cb.shape[0], scale, 0.0, out.data_ptr(), ws.data_ptr(), ws.numel(),
                           D.stream_handle(a.device)), "q_e8 search only")
    return out.cpu().numpy()


def _torch_nearest(gn, cb, chunk=4096):
    """Exact nearest codeword by fp64 distances on the device (torch), lowest
    index on ties (argmin's first index)."""
    import torch
    x = torch.from_numpy(gn).cuda()
    c = torch.from_numpy(cb).cuda()
    idx = []
    for s in range(0, x.shape[0], chunk):
        xb = x[s:s + chunk]
        d = torch.zeros((xb.shape[0], c.shape[0]), dtype=torch.float64, device=x.device)
        for i in range(8):
            e = xb[:, i:i + 1] - c[None, :, i]
            d = d + e * e
        idx.append(torch.argmin(d, dim=1))
    return torch.cat(idx).cpu().numpy()


def test_q_e8_large_vs_brute_force(uq):
    """256 x 4096 Student-t at 2 bpw (131,072 vectors, K = 65,536): the lattice
    shortcut and the search agree bit for bit, and both equal the exact
    nearest codeword from an fp64 brute force."""
    rng = np.random.RandomState(8)
    A = rng.standard_t(4, size=(256, 4096)) * 0.02
    got = uq.q_e8(A, 2.0)
    assert same_bits(got, _search_only(uq, A, 2.0))
    g = A.reshape(-1, 256)
    s = np.sqrt((g ** 2).mean(1, keepdims=True)) + 1e-12
    gn = (g / s).reshape(-1, 8)
    cb = uq.e8_codebook(65536)
    ref = (cb[_torch_nearest(gn, cb)].reshape(-1, 256) * s).reshape(A.shape)
    assert same_bits(got, ref)


def test_q_e8_edges(uq):
    """Empty input, non-finite input (cKDTree's ValueError), fp32 input."""
    assert uq.q_e8(np.zeros((0, 256)), 2.0).shape == (0, 256)
    bad = np.zeros((2, 256))
    bad[1, 3] = np.nan
    with pytest.raises(ValueError, match="finite"):
        uq.q_e8(bad, 2.0)
    rng = np.random.RandomState(5)
    A = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    assert same_bits(uq.q_e8(A, 2.0), O.q_e8(A, 2.0))
