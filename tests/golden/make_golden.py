#!/usr/bin/env python
"""Generate the golden fixtures for the quantization hot path.

Runs the *reference* modules (qlab.py, trellis.py, qat.py of
hackerbbrine/UltraQuant) on small seeded inputs, on the CPU, and stores inputs
and outputs in ``tests/golden/*.npz``.  The reference has no test suite and no
committed golden vectors; these fixtures pin the oracle and the CUDA path.

Usage (in a container that has the reference checkout):
    python tests/golden/make_golden.py /path/to/reference [rht e8 trellis pipeline qat ...]
or with UQ_REFERENCE=/path/to/reference and no positional path.

Nothing at test or bench time reads the reference; only this generator does.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("UQ_REFERENCE", "")
if not REF and __name__ == "__main__":
    sys.exit("usage: make_golden.py /path/to/reference [makers...]  (or set UQ_REFERENCE)")


def _import_reference():
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, REF)
    import qlab  # noqa: E402
    import trellis  # noqa: E402
    import qat  # noqa: E402
    qat.DEV = "cpu"  # read at call time (qat.py:9)
    return qlab, trellis, qat


def _versions():
    import scipy
    import torch
    return np.array(f"numpy={np.__version__} scipy={scipy.__version__} torch={torch.__version__}")


def student_t(rng, shape, nu=4.0, std=0.02):
    x = rng.standard_t(nu, size=shape)
    return (x / np.sqrt(nu / (nu - 2.0)) * std)


def gauss_outliers(rng, shape, std=0.02, frac=0.001):
    x = rng.normal(0.0, std, size=shape)
    m = rng.random_sample(shape) < frac
    x[m] = np.sign(rng.normal(size=m.sum())) * 8 * std
    return x


def make_rht(qlab):
    rng = np.random.RandomState(11)
    out = {"versions": _versions()}
    for n in [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768]:
        out[f"signs_{n}"] = np.random.RandomState(0).choice([-1.0, 1.0], size=n).astype(np.int8)
    out["signs_seed7_1024"] = np.random.RandomState(7).choice([-1.0, 1.0], size=1024).astype(np.int8)
    cases = [
        ("a", rng.randn(5, 300), 0),                      # pad 300 -> 512
        ("b", rng.randn(2, 4096) * 0.02, 0),              # exact pow2
        ("c", rng.randn(4, 1000).astype(np.float32), 0),  # float32 input
        ("d", rng.randn(2, 1), 0),                        # n0 = 1 -> n = 1
        ("e", rng.randn(3, 24), 0),                       # tiny
        ("f", rng.randn(1, 5000), 7),                     # other seed, pad to 8192
        ("g", np.zeros((0, 64)), 0),                      # no rows
        ("h", rng.randn(1, 16384) * 1e-3, 0),             # ffn_down padded width
        ("i", gauss_outliers(rng, (2, 2048)), 0),
    ]
    for tag, A, seed in cases:
        X = qlab.rht_rows(A, seed=seed)
        out[f"rht_{tag}_in"] = A
        out[f"rht_{tag}_seed"] = np.array(seed)
        out[f"rht_{tag}_out"] = X
        out[f"irht_{tag}_out"] = qlab.irht_rows(X, A.shape[1], seed=seed)
        if tag in ("a", "c", "e", "f"):
            out[f"irht_{tag}_f32_out"] = qlab.irht_rows(X.astype(np.float32), A.shape[1], seed=seed)
    np.savez_compressed(os.path.join(HERE, "golden_rht.npz"), **out)


def make_e8(qlab):
    rng = np.random.RandomState(12)
    out = {"versions": _versions()}
    Y = np.concatenate([
        rng.randn(1500, 8) * 2.5,
        rng.randn(500, 8) * 40.0,
        np.round(rng.randn(200, 8) * 3),                      # integers (odd sums keep parity)
        np.round(rng.randn(200, 8) * 3) + 0.5,                # half-integers: rounding ties
        np.round(rng.randn(100, 8) * 4) / 2,                  # mixed ties
        np.zeros((4, 8)),
    ])
    out["Y"] = Y
    out["d8"] = qlab._d8_decode(Y.copy())
    out["e8"] = qlab.e8_decode(Y)
    pts = qlab.e8_decode(rng.randn(4000, 8) * 1.3)
    out["ent_pts"] = pts
    out["ent_bpw"] = np.array(qlab._entropy_bpw(pts))
    A = student_t(rng, (8, 1024), std=0.015)
    out["q_A"] = A
    for step in (0.48, 0.25, 0.16, 0.11):
        out[f"q_fixed_{step}"] = qlab.q_e8_fast(A, fixed_step=step)
    A2 = rng.randn(3, 100)                                    # size not a multiple of the group
    out["q_A2"] = A2
    out["q_A2_fixed_0.48"] = qlab.q_e8_fast(A2, fixed_step=0.48)
    out["q_A2_g64_fixed_0.25"] = qlab.q_e8_fast(A2, group=64, fixed_step=0.25)
    A3 = student_t(rng, (16, 2048), std=0.02)
    out["q_A3"] = A3
    for tb in (2.0, 3.0):
        qlab._E8_SCALE.clear()
        rec = qlab.q_e8_fast(A3, target_bpw=tb, calib_key="k")
        out[f"q_cal_{tb}_step"] = np.array(qlab._E8_SCALE["k"])
        out[f"q_cal_{tb}_rec"] = rec
    qlab._E8_SCALE.clear()
    np.savez_compressed(os.path.join(HERE, "golden_e8.npz"), **out)


def make_trellis(trellis, qat):
    rng = np.random.RandomState(13)
    out = {"versions": _versions()}
    out["codebook16"] = trellis.codebook(16)
    out["pred_8_2"] = trellis.pred_table(8, 2)
    cases = [
        # tag, shape, L, R, seg, group
        ("l8r2", (8, 512), 8, 2, 64, 256),
        ("l8r1", (4, 512), 8, 1, 64, 256),
        ("l8r3", (4, 512), 8, 3, 64, 256),
        ("l8r4", (4, 512), 8, 4, 64, 256),
        ("l10r2", (4, 512), 10, 2, 128, 256),
        ("l12r2", (8, 512), 12, 2, 256, 256),
        ("l12r2s64", (4, 512), 12, 2, 64, 256),
        ("l12r3", (2, 512), 12, 3, 256, 256),
        ("l16r2", (1, 512), 16, 2, 256, 256),
        ("l16r3", (1, 512), 16, 3, 256, 256),
        ("pad", (3, 100), 8, 2, 64, 256),                 # 300 weights -> padded to 512
        ("g128", (2, 384), 10, 2, 64, 128),
    ]
    for tag, shape, L, R, seg, group in cases:
        A = gauss_outliers(rng, shape, std=1.0).astype(np.float32)
        rec = trellis.trellis_quant_fast(A, L=L, R=R, seg=seg, scale_group=group, device="cpu")
        st, sc_g, cw, meta = qat.trellis_encode(A, L=L, R=R, seg=seg, scale_group=group)
        out[f"tq_{tag}_in"] = A
        out[f"tq_{tag}_cfg"] = np.array([L, R, seg, group])
        out[f"tq_{tag}_rec"] = rec
        out[f"tq_{tag}_states"] = st
        out[f"tq_{tag}_scg"] = sc_g
    # full-row Viterbi (trellis.py:27-60)
    for tag, shape, L, R, group in [("r8", (3, 300), 8, 2, 256), ("r10", (2, 256), 10, 2, 128)]:
        A = rng.randn(*shape).astype(np.float32)
        out[f"tr_{tag}_in"] = A
        out[f"tr_{tag}_cfg"] = np.array([L, R, group])
        out[f"tr_{tag}_rec"] = trellis.trellis_quant(A, L=L, R=R, group=group, chunk_rows=512, device="cpu")
    # self-test KAT (trellis.py:110-117) on a reduced unit-Gaussian
    X = np.random.RandomState(0).randn(64, 1024).astype(np.float32)
    Xh = trellis.trellis_quant(X, L=8, R=2, group=256, chunk_rows=64, device="cpu")
    out["selftest_l8_nmse"] = np.array(float(np.sum((X - Xh) ** 2) / np.sum(X ** 2)))
    np.savez_compressed(os.path.join(HERE, "golden_trellis.npz"), **out)


def make_pipeline(qlab, trellis, qat):
    import torch
    rng = np.random.RandomState(14)
    out = {"versions": _versions()}
    W = student_t(rng, (16, 300), std=0.02)
    H = np.exp(rng.normal(0.0, 1.0, size=300))
    out["W"] = W
    out["H"] = H
    # buildtrellis.py:16-20 recipe, through the reference functions
    for L, R, seg in [(8, 2, 64), (12, 2, 64), (10, 3, 256)]:
        Hc = np.maximum(H, H.max() * 1e-3)
        sH = np.sqrt(Hc)[None, :]
        A = W * sH
        Arot = qlab.rht_rows(A)
        rec = trellis.trellis_quant_fast(Arot, L=L, R=R, seg=seg, scale_group=256, mem_gb=4.0, device="cpu")
        Ah = qlab.irht_rows(rec, A.shape[1])
        out[f"qt_{L}_{R}_{seg}_What"] = (Ah / sH).astype(np.float32)
        out[f"qt_{L}_{R}_{seg}_wnmse"] = np.array(qlab.wnmse(A, Ah))
    # buildalloc.py:21-24 recipe
    for step in (0.48, 0.25):
        Hc = np.maximum(H, H.max() * 1e-3)
        sH = np.sqrt(Hc)[None, :]
        Ah = qlab.irht_rows(qlab.q_e8_fast(qlab.rht_rows(W * sH), fixed_step=step), W.shape[1])
        out[f"qs_{step}_What"] = (Ah / sH).astype(np.float32)
    # qat.py:61-89 decoder path: states -> recon_torch (fixed cw, sc_g)
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = qlab.rht_rows(W * sH).astype(np.float32)
    st, sc_g, cwn, meta = qat.trellis_encode(A, L=8, R=2, seg=64, scale_group=256)
    cw = torch.tensor(cwn)
    Wh = qat.recon_torch(st, cw, torch.tensor(sc_g), meta, torch.tensor(sH, dtype=torch.float32), 300)
    out["qat_states"] = st
    out["qat_scg"] = sc_g
    out["qat_recon"] = Wh.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_pipeline.npz"), **out)


def make_qat(qlab, qat):
    """qat.py:35-59: fwht_torch / irht_torch / recon_torch values and the
    gradients torch's autograd gives for loss = sum(out * U)."""
    import torch
    rng = np.random.RandomState(15)
    out = {"versions": _versions()}

    def grads(fn, x, shape_out):
        x = x.clone().requires_grad_(True)
        y = fn(x)
        U = torch.from_numpy(rng.normal(size=shape_out).astype(np.float32)).to(x.dtype)
        (y * U).sum().backward()
        return y.detach().numpy(), U.numpy(), x.grad.numpy()

    for dt in ("f32", "f64"):
        tdt = torch.float32 if dt == "f32" else torch.float64
        for n in (1, 2, 8, 32, 256, 512, 4096, 8192):
            rows = 3 if n <= 512 else 1
            x = torch.from_numpy(rng.normal(size=(rows, n))).to(tdt)
            y, U, g = grads(qat.fwht_torch, x, (rows, n))
            out[f"fwht_{dt}_{n}_x"], out[f"fwht_{dt}_{n}_y"] = x.numpy(), y
            out[f"fwht_{dt}_{n}_U"], out[f"fwht_{dt}_{n}_gx"] = U, g
        for n, in0 in ((512, 300), (4096, 4096), (4096, 2999), (16384, 14336)):
            if n == 16384 and dt == "f64":
                continue
            rows = 1 if n >= 4096 else 4
            x = torch.from_numpy(rng.normal(size=(rows, n))).to(tdt)
            y, U, g = grads(lambda t: qat.irht_torch(t, in0), x, (rows, in0))
            key = f"irht_{dt}_{n}_{in0}"
            out[key + "_x"], out[key + "_y"], out[key + "_U"], out[key + "_gx"] = x.numpy(), y, U, g
    # recon_torch from the reference encoder (fixed states), forward and
    # gradients with respect to cw and sc_g
    cases = [("a", 8, 300, 8, 2, 64), ("b", 3, 128, 6, 2, 64), ("c", 16, 1000, 10, 3, 256)]
    for tag, rows, n0, L, R, seg in cases:
        W = student_t(rng, (rows, n0), std=0.02)
        H = np.exp(rng.normal(0.0, 1.0, size=n0))
        Hc = np.maximum(H, H.max() * 1e-3)
        sH = np.sqrt(Hc)[None, :]
        A = qlab.rht_rows(W * sH).astype(np.float32)
        st, sc_g, cwn, meta = qat.trellis_encode(A, L=L, R=R, seg=seg, scale_group=256)
        cw = torch.tensor(cwn, requires_grad=True)
        scg = torch.tensor(sc_g, requires_grad=True)
        sH_t = torch.tensor(sH, dtype=torch.float32)
        Wh = qat.recon_torch(st, cw, scg, meta, sH_t, n0)
        U = torch.from_numpy(rng.normal(size=Wh.shape).astype(np.float32))
        (Wh * U).sum().backward()
        key = f"recon_{tag}"
        out[key + "_states"], out[key + "_scg"], out[key + "_sH"] = st, sc_g, sH.astype(np.float32)
        out[key + "_meta"] = np.array([meta[k] for k in ("nrow", "ncol", "Ntot", "seg", "scale_group",
                                                         "pad", "Nseg")] + [L, n0])
        out[key + "_What"], out[key + "_U"] = Wh.detach().numpy(), U.numpy()
        out[key + "_gcw"], out[key + "_gsc"] = cw.grad.numpy(), scg.grad.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_qat.npz"), **out)


def make_q8(qlab):
    """buildq.py:21-30 enc_q8 and qlab.py:27-32 deq_q8 on seeded matrices with
    zero blocks, exact halves, huge and tiny magnitudes; the encoder is
    imported from the reference builder module."""
    import importlib
    buildq = importlib.import_module("buildq")
    rng = np.random.RandomState(16)
    out = {"versions": _versions()}
    W = rng.normal(0, 0.02, size=(24, 1024)).astype(np.float32)
    W[3, :32] = 0.0                                    # zero block -> scale 1e-9
    W[4, :64] = np.arange(64) - 31.5                  # many x / sc near .5
    W[5, 32:64] = 127.0 * np.array([k / 127.0 for k in range(32)], np.float32)
    W[6] *= 1e4
    W[7] *= 1e-6
    W[8, ::2] = -W[8, 1::2]
    W64 = rng.standard_t(4, size=(8, 256)) * 0.02
    for tag, M in (("f32", W), ("f64", W64)):
        q = buildq.enc_q8(M)

        class _T:
            data = q
        out[f"q8_{tag}_W"] = M
        out[f"q8_{tag}_enc"] = q
        out[f"q8_{tag}_dec"] = qlab.deq_q8(_T())
    np.savez_compressed(os.path.join(HERE, "golden_q8.npz"), **out)


def make_quniform(qlab):
    """qlab.py:100-106 q_uniform on fp64 and fp32 matrices at several rates."""
    rng = np.random.RandomState(17)
    out = {"versions": _versions()}
    A = rng.standard_t(4, size=(16, 256)) * 0.02
    A[2, :32] = 0.0
    A[3, :32] = np.arange(32) / 31.0 - 0.5
    for tag, M in (("f64", A), ("f32", A.astype(np.float32))):
        out[f"qu_{tag}_A"] = M
        for bpw in (2, 3, 4, 2.5):
            with np.errstate(invalid="ignore"):
                out[f"qu_{tag}_{bpw}"] = qlab.q_uniform(M, bpw)
        out[f"qu_{tag}_bs64"] = qlab.q_uniform(M, 3, bs=64)
    np.savez_compressed(os.path.join(HERE, "golden_quniform.npz"), **out)


def make_qe8(qlab):
    """qlab.py:185-198 q_e8 (cKDTree nearest codeword) at three rates, fp32
    input, another group size, a ragged size and edge rows; fingerprints of
    e8_codebook (qlab.py:111-124) for several K."""
    import hashlib
    rng = np.random.RandomState(21)
    out = {"versions": _versions()}
    Ks = np.array([16, 256, 4096, 65536, 1 << 20], np.int64)
    out["cb_K"] = Ks
    out["cb_sha256"] = np.array([hashlib.sha256(qlab.e8_codebook(int(K)).tobytes()).hexdigest() for K in Ks])
    out["cb_256"] = qlab.e8_codebook(256)
    A = student_t(rng, (16, 512), std=0.02)
    out["qe_A"] = A
    for bpw in (1.0, 1.5, 2.0):
        out[f"qe_A_{bpw}"] = qlab.q_e8(A, bpw)
    out["qe_A32_2.0"] = qlab.q_e8(A.astype(np.float32), 2.0)
    out["qe_A_g64_2.0"] = qlab.q_e8(A[:8], 2.0, group_scale=64)
    R = rng.standard_normal((7, 100))
    out["qe_R"] = R
    out["qe_R_2.0"] = qlab.q_e8(R, 2.0)
    E = student_t(rng, (6, 256), std=0.02)
    E[0] = 0.0                       # zero group
    E[1, :] = 0.0
    E[1, 7] = 5.0                    # one outlier in a group
    E[2] = 0.013                     # constant group
    E[3] *= 1e-200                   # tiny values
    E[4, ::2] = 0.0                  # half zeros
    out["qe_E"] = E
    out["qe_E_2.0"] = qlab.q_e8(E, 2.0)
    np.savez_compressed(os.path.join(HERE, "golden_qe8.npz"), **out)


MAKERS = {"rht": lambda m: make_rht(m[0]), "e8": lambda m: make_e8(m[0]),
          "trellis": lambda m: make_trellis(m[1], m[2]), "pipeline": lambda m: make_pipeline(*m),
          "qat": lambda m: make_qat(m[0], m[2]), "q8": lambda m: make_q8(m[0]),
          "quniform": lambda m: make_quniform(m[0]), "qe8": lambda m: make_qe8(m[0])}


def main():
    mods = _import_reference()
    which = sys.argv[2:] or list(MAKERS)
    for name in which:
        MAKERS[name](mods)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
