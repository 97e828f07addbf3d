"""GPU parity of the differentiable QAT decoder (qat.py:35-59): fwht_torch,
irht_torch and recon_torch, forward values and autograd gradients, against
the reference goldens and the oracle."""
import numpy as np
import pytest

import oracle as O
from conftest import grad_close, qat_meta, same_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Q():
    import ultraquant_b200.qat as Q
    return Q


def _fwd_bwd(fn, x, U, dev="cuda"):
    import torch
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(dev).requires_grad_(True)
    y = fn(xt)
    (y * torch.from_numpy(np.ascontiguousarray(U)).to(dev)).sum().backward()
    return y.detach().cpu().numpy(), xt.grad.cpu().numpy()


@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_fwht_irht_golden(Q, g_qat, dt):
    for n in (1, 2, 8, 32, 256, 512, 4096, 8192):
        k = f"fwht_{dt}_{n}"
        y, gx = _fwd_bwd(Q.fwht_torch, g_qat[k + "_x"], g_qat[k + "_U"])
        assert same_bits(y, g_qat[k + "_y"]), k
        assert same_bits(gx, g_qat[k + "_gx"]), k
    for n, in0 in ((512, 300), (4096, 4096), (4096, 2999), (16384, 14336)):
        k = f"irht_{dt}_{n}_{in0}"
        if k + "_x" not in g_qat:
            continue
        y, gx = _fwd_bwd(lambda t: Q.irht_torch(t, in0), g_qat[k + "_x"], g_qat[k + "_U"])
        assert same_bits(y, g_qat[k + "_y"]), k
        assert same_bits(gx, g_qat[k + "_gx"]), k


@pytest.mark.parametrize("dt,n,rows", [("f32", 16384, 3), ("f32", 32768, 2), ("f64", 16384, 2),
                                       ("f32", 64, 1000), ("f64", 2048, 37)])
def test_fwht_irht_vs_oracle(Q, dt, n, rows):
    """Sizes beyond the goldens (n = 32768 for f32) and many rows per tile."""
    rng = np.random.RandomState(n + rows)
    npdt = np.float32 if dt == "f32" else np.float64
    x = rng.normal(size=(rows, n)).astype(npdt)
    U = rng.normal(size=(rows, n)).astype(npdt)
    y, gx = _fwd_bwd(Q.fwht_torch, x, U)
    yr, gr = _fwd_bwd(O.fwht_torch, x, U, dev="cpu")
    assert same_bits(y, yr) and same_bits(gx, gr)
    in0 = n - n // 7
    Ui = np.ascontiguousarray(U[:, :in0])
    y, gx = _fwd_bwd(lambda t: Q.irht_torch(t, in0), x, Ui)
    yr, gr = _fwd_bwd(lambda t: O.irht_torch(t, in0), x, Ui, dev="cpu")
    assert same_bits(y, yr) and same_bits(gx, gr)


def test_fwht_cpu_tensor_and_shapes(Q):
    """CPU tensors come back on the CPU; leading dimensions are kept."""
    import torch
    x = torch.randn(2, 3, 256, dtype=torch.float64)
    y = Q.fwht_torch(x)
    assert y.device.type == "cpu" and y.shape == x.shape
    assert same_bits(y.numpy(), O.fwht_torch(x).numpy())
    with pytest.raises(RuntimeError):
        Q.fwht_torch(torch.zeros(4, 12, device="cuda"))
    with pytest.raises(NotImplementedError):
        Q.fwht_torch(torch.zeros(4, 16, dtype=torch.float16, device="cuda"))


def _recon(Q, g, tag, states=None):
    import torch
    k = f"recon_{tag}"
    meta, L, in0 = qat_meta(g, k)
    cw = torch.tensor(O.codebook(L), device="cuda", requires_grad=True)
    scg = torch.tensor(g[k + "_scg"], device="cuda", requires_grad=True)
    sH = torch.tensor(g[k + "_sH"], device="cuda")
    st = g[k + "_states"] if states is None else states
    Wh = Q.recon_torch(st, cw, scg, meta, sH, in0)
    return k, meta, L, in0, cw, scg, Wh


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_recon_golden(Q, g_qat, tag):
    import torch
    k, meta, L, in0, cw, scg, Wh = _recon(Q, g_qat, tag)
    assert same_bits(Wh.detach().cpu().numpy(), g_qat[k + "_What"])
    (Wh * torch.from_numpy(g_qat[k + "_U"]).cuda()).sum().backward()
    from test_oracle_golden import recon_exact_grads
    gcw, gsc = recon_exact_grads(g_qat[k + "_states"], O.codebook(L), g_qat[k + "_scg"], g_qat[k + "_U"],
                                 meta, g_qat[k + "_sH"], in0)
    assert grad_close(cw.grad.cpu().numpy(), g_qat[k + "_gcw"], gcw)
    assert grad_close(scg.grad.cpu().numpy().reshape(-1), g_qat[k + "_gsc"].reshape(-1), gsc)
    assert scg.grad.shape == scg.shape


def test_recon_int64_states_and_device_states(Q, g_qat):
    import torch
    k = "recon_a"
    st64 = torch.from_numpy(g_qat[k + "_states"].astype(np.int64)).cuda()
    *_, Wh = _recon(Q, g_qat, "a", states=st64)
    assert same_bits(Wh.detach().cpu().numpy(), g_qat[k + "_What"])


def test_recon_state_out_of_range(Q, g_qat):
    """Host states are checked before launch; device states are bounds-checked
    in the kernel (no access outside the codebook), give NaN and are reported."""
    import torch
    from ultraquant_b200 import _lib, _device as D
    bad = g_qat["recon_a_states"].copy()
    bad[1, 5] = 1 << 8
    with pytest.raises(IndexError):
        _recon(Q, g_qat, "a", states=bad)
    *_, Wh = _recon(Q, g_qat, "a", states=torch.from_numpy(bad).cuda())
    lib = _lib.load()
    rc = lib.uq_device_errors(D.stream_handle())
    assert rc == _lib.UQ_ERR_INVALID
    assert torch.isnan(Wh).any()
    assert lib.uq_device_errors(D.stream_handle()) == _lib.UQ_OK   # cleared


def test_recon_full_size_vs_oracle(Q):
    """4096 x 4096 at L = 16 (the headline tensor shape): forward bit-exact
    against the oracle; gradients against the fp64 restatement."""
    import torch
    from test_oracle_golden import recon_exact_grads
    rng = np.random.RandomState(3)
    nrow = n = 4096
    L = 16
    states = rng.randint(0, 1 << L, size=(nrow * n // 256, 256)).astype(np.int32)
    scg = (np.abs(rng.normal(size=(nrow * n // 256, 1))) + 0.1).astype(np.float32)
    sH = np.sqrt(np.maximum(np.exp(rng.normal(size=(1, n))), 1e-3)).astype(np.float32)
    meta = dict(nrow=nrow, ncol=n, Ntot=nrow * n, seg=256, scale_group=256, pad=0, Nseg=states.shape[0])
    cwn = O.codebook(L)
    cw = torch.tensor(cwn, device="cuda", requires_grad=True)
    sc = torch.tensor(scg, device="cuda", requires_grad=True)
    Wh = Q.recon_torch(states, cw, sc, meta, torch.tensor(sH, device="cuda"), n)
    ref = O.recon_torch(states, torch.tensor(cwn), torch.tensor(scg), meta, torch.tensor(sH), n)
    assert same_bits(Wh.detach().cpu().numpy(), ref.numpy())
    U = rng.normal(size=(nrow, n)).astype(np.float32)
    (Wh * torch.from_numpy(U).cuda()).sum().backward()
    gcw, gsc = recon_exact_grads(states, cwn, scg, U, meta, sH, n)
    assert grad_close(cw.grad.cpu().numpy(), gcw, gcw)
    assert grad_close(sc.grad.cpu().numpy().reshape(-1), gsc, gsc)


def test_qat_loop_runs_through_dropin(Q, g_qat):
    """qat.py:73-79: Adam steps on (cw, sc_g) through recon_torch reduce the
    output error as the reference's loop does."""
    import torch
    k = "recon_c"
    meta, L, in0 = qat_meta(g_qat, k)
    rng = np.random.RandomState(5)
    Wt = torch.from_numpy(g_qat[k + "_What"]).cuda() + 0.01 * torch.from_numpy(
        rng.normal(size=g_qat[k + "_What"].shape).astype(np.float32)).cuda()
    X = torch.from_numpy(rng.normal(size=(64, in0)).astype(np.float32)).cuda()
    target = X @ Wt.T
    cw = torch.tensor(O.codebook(L), device="cuda", requires_grad=True)
    scg = torch.tensor(g_qat[k + "_scg"], device="cuda", requires_grad=True)
    sH = torch.tensor(g_qat[k + "_sH"], device="cuda")
    opt = torch.optim.Adam([cw, scg], lr=2e-3)

    def loss():
        return ((X @ Q.recon_torch(g_qat[k + "_states"], cw, scg, meta, sH, in0).T - target) ** 2).mean()

    l0 = loss().item()
    for _ in range(20):
        opt.zero_grad()
        ls = loss()
        ls.backward()
        opt.step()
    assert loss().item() < l0


@pytest.mark.parametrize("nrow,n,L,in0", [(64, 4096, 12, 4096), (24, 8192, 12, 7000), (8, 16384, 10, 14336),
                                          (16, 8192, 16, 8192)])
def test_recon_widths_vs_oracle(Q, nrow, n, L, in0):
    """The row-layout decoder at 4096 / 8192 / 16384 columns, codebooks in
    shared memory (L <= 12) and in global memory (L = 16), cropped widths:
    forward bit-exact against the oracle, gradients against the fp64
    restatement."""
    import torch
    from test_oracle_golden import recon_exact_grads
    rng = np.random.RandomState(nrow + n + L)
    states = rng.randint(0, 1 << L, size=(nrow * n // 256, 256)).astype(np.int32)
    scg = (np.abs(rng.normal(size=(nrow * n // 256, 1))) + 0.1).astype(np.float32)
    sH = np.sqrt(np.maximum(np.exp(rng.normal(size=(1, in0))), 1e-3)).astype(np.float32)
    meta = dict(nrow=nrow, ncol=n, Ntot=nrow * n, seg=256, scale_group=256, pad=0, Nseg=states.shape[0])
    cwn = O.codebook(L)
    cw = torch.tensor(cwn, device="cuda", requires_grad=True)
    sc = torch.tensor(scg, device="cuda", requires_grad=True)
    Wh = Q.recon_torch(states, cw, sc, meta, torch.tensor(sH, device="cuda"), in0)
    ref = O.recon_torch(states, torch.tensor(cwn), torch.tensor(scg), meta, torch.tensor(sH), in0)
    assert same_bits(Wh.detach().cpu().numpy(), ref.numpy())
    U = rng.normal(size=(nrow, in0)).astype(np.float32)
    (Wh * torch.from_numpy(U).cuda()).sum().backward()
    gcw, gsc = recon_exact_grads(states, cwn, scg, U, meta, sH, in0)
    assert grad_close(cw.grad.cpu().numpy(), gcw, gcw)
    assert grad_close(sc.grad.cpu().numpy().reshape(-1), gsc, gsc)
