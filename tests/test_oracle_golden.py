"""Pin the CPU oracle against golden vectors produced by the reference itself."""
import numpy as np
import pytest

import oracle as O
from conftest import qe8_same_or_tie, same_bits


def test_signs(g_rht):
    for n in [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768]:
        assert np.array_equal(O.rht_signs(n).astype(np.int8), g_rht[f"signs_{n}"])
    assert np.array_equal(O.rht_signs(1024, 7).astype(np.int8), g_rht["signs_seed7_1024"])


@pytest.mark.parametrize("tag", list("abcdefghi"))
def test_rht_irht(g_rht, tag):
    A = g_rht[f"rht_{tag}_in"]
    seed = int(g_rht[f"rht_{tag}_seed"])
    X = O.rht_rows(A, seed=seed)
    assert same_bits(X, g_rht[f"rht_{tag}_out"])
    assert same_bits(O.irht_rows(X, A.shape[1], seed=seed), g_rht[f"irht_{tag}_out"])
    k = f"irht_{tag}_f32_out"
    if k in g_rht:
        assert same_bits(O.irht_rows(X.astype(np.float32), A.shape[1], seed=seed), g_rht[k])


def test_d8_e8(g_e8):
    Y = g_e8["Y"]
    assert same_bits(O.d8_decode(Y.copy()), g_e8["d8"])
    assert same_bits(O.e8_decode(Y), g_e8["e8"])


def test_entropy(g_e8):
    assert O.entropy_bpw(g_e8["ent_pts"]) == float(g_e8["ent_bpw"])


def test_q_e8_fixed(g_e8):
    A = g_e8["q_A"]
    for step in (0.48, 0.25, 0.16, 0.11):
        assert same_bits(O.q_e8_fast(A, fixed_step=step), g_e8[f"q_fixed_{step}"])
    A2 = g_e8["q_A2"]
    assert same_bits(O.q_e8_fast(A2, fixed_step=0.48), g_e8["q_A2_fixed_0.48"])
    assert same_bits(O.q_e8_fast(A2, group=64, fixed_step=0.25), g_e8["q_A2_g64_fixed_0.25"])


@pytest.mark.parametrize("tb", [2.0, 3.0])
def test_q_e8_calibrated(g_e8, tb):
    cache = {}
    rec = O.q_e8_fast(g_e8["q_A3"], target_bpw=tb, calib_key="k", cache=cache)
    assert cache["k"] == float(g_e8[f"q_cal_{tb}_step"])
    assert same_bits(rec, g_e8[f"q_cal_{tb}_rec"])


def test_codebook(g_trellis):
    cb = O.codebook(16)
    assert same_bits(cb, g_trellis["codebook16"])
    # smaller L are prefixes of the L=16 table (the hash depends on s only)
    assert same_bits(O.codebook(12), cb[:4096])
    assert np.array_equal(O.pred_table(8, 2), g_trellis["pred_8_2"])


TQ = ["l8r2", "l8r1", "l8r3", "l8r4", "l10r2", "l12r2", "l12r2s64", "l12r3", "l16r2",
      "l16r3", "pad", "g128"]


@pytest.mark.parametrize("tag", TQ)
def test_trellis_fast_and_encode(g_trellis, tag):
    A = g_trellis[f"tq_{tag}_in"]
    L, R, seg, group = (int(v) for v in g_trellis[f"tq_{tag}_cfg"])
    if L == 16:
        pytest.importorskip("torch")
    rec = O.trellis_quant_fast(A, L=L, R=R, seg=seg, scale_group=group)
    assert same_bits(rec, g_trellis[f"tq_{tag}_rec"])
    st, sc_g, cw, meta = O.trellis_encode(A, L=L, R=R, seg=seg, scale_group=group)
    assert np.array_equal(st, g_trellis[f"tq_{tag}_states"])
    assert same_bits(sc_g, g_trellis[f"tq_{tag}_scg"])
    assert same_bits(O.trellis_decode(st, cw, sc_g, meta), rec)


@pytest.mark.parametrize("tag", TQ)
def test_c_viterbi_golden(g_trellis, tag):
    """The C restatement of the Viterbi (oracle/uq_viterbi_ref.c) returns the
    reference's state paths on every golden configuration."""
    from oracle import cviterbi as CV
    from oracle.uq_oracle import _flat_normalise
    A = g_trellis[f"tq_{tag}_in"]
    L, R, seg, group = (int(v) for v in g_trellis[f"tq_{tag}_cfg"])
    xn, _, _, _ = _flat_normalise(A, seg, group)
    assert np.array_equal(CV.viterbi_segments_c(xn, L, R), g_trellis[f"tq_{tag}_states"])


@pytest.mark.parametrize("L,R,T", [(6, 1, 32), (8, 4, 64), (11, 3, 256), (12, 2, 1), (12, 2, 2), (14, 2, 64),
                                   (16, 2, 64), (16, 3, 32)])
def test_c_viterbi_vs_torch_restatement(L, R, T):
    """C and torch restatements agree on random and tie-provoking sequences;
    the fp32 path cost of the C path equals the minimum final cost."""
    from oracle import cviterbi as CV
    rng = np.random.RandomState(L * 100 + R * 10 + T)
    x = rng.randn(6, T).astype(np.float32)
    x[:3] = np.round(x[:3] * 2) / 2
    st = CV.viterbi_segments_c(x, L, R, threads=2)
    assert np.array_equal(st, O.viterbi_segments(x, L, R))
    # the path cost matches an independent evaluation of the same recurrence
    cw = O.codebook(L)
    acc = np.zeros(6, np.float32)
    for t in range(T):
        d = (x[:, t] - cw[st[:, t]]).astype(np.float32)
        acc = (d * d + acc).astype(np.float32) if t else (d * d).astype(np.float32)
    assert np.array_equal(CV.path_costs(x, st, L).view(np.int32), acc.view(np.int32))


def test_product_pred_table(g_trellis):
    """ultraquant_b200.trellis.pred_table (trellis.py:21-25) against the
    reference's table and the oracle, for every (L, R) the Viterbi builds."""
    from ultraquant_b200 import trellis as T
    assert np.array_equal(T.pred_table(8, 2), g_trellis["pred_8_2"])
    for L, R in [(6, 1), (8, 3), (10, 2), (12, 2), (12, 4), (16, 2), (16, 3)]:
        p = T.pred_table(L, R)
        assert p.shape == (1 << L, 1 << R)
        assert np.array_equal(p, O.pred_table(L, R))
        # every state's predecessors shift into it: ((pred << R) | (s & mask)) mod 2^L == s
        s = np.arange(1 << L)[:, None]
        assert np.array_equal(((p << R) | (s & ((1 << R) - 1))) & ((1 << L) - 1), np.broadcast_to(s, p.shape))


@pytest.mark.parametrize("tag", ["r8", "r10"])
def test_trellis_full_row(g_trellis, tag):
    A = g_trellis[f"tr_{tag}_in"]
    L, R, group = (int(v) for v in g_trellis[f"tr_{tag}_cfg"])
    assert same_bits(O.trellis_quant(A, L=L, R=R, group=group), g_trellis[f"tr_{tag}_rec"])


def test_selftest_kat(g_trellis):
    X = np.random.RandomState(0).randn(64, 1024).astype(np.float32)
    Xh = O.trellis_quant(X, L=8, R=2, group=256)
    nmse = float(np.sum((X - Xh) ** 2) / np.sum(X ** 2))
    assert nmse == float(g_trellis["selftest_l8_nmse"])
    # trellis.py:110-117 / FINDINGS: L=8 R=2 beats memoryless (~0.118), above 2^-4
    assert 0.0625 < nmse < 0.118


def test_pipelines(g_pipeline):
    import torch
    W, H = g_pipeline["W"], g_pipeline["H"]
    for L, R, seg in [(8, 2, 64), (12, 2, 64), (10, 3, 256)]:
        Wh = O.quant_trellis(W, H, L=L, R=R, seg=seg)
        assert same_bits(Wh, g_pipeline[f"qt_{L}_{R}_{seg}_What"])
    for step in (0.48, 0.25):
        assert same_bits(O.quant_step(W, H, step), g_pipeline[f"qs_{step}_What"])
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = O.rht_rows(W * sH).astype(np.float32)
    st, sc_g, cwn, meta = O.trellis_encode(A, L=8, R=2, seg=64, scale_group=256)
    assert np.array_equal(st, g_pipeline["qat_states"])
    Wh = O.recon_torch(st, torch.tensor(cwn), torch.tensor(sc_g), meta,
                       torch.tensor(sH, dtype=torch.float32), 300)
    assert same_bits(Wh.numpy(), g_pipeline["qat_recon"])


# ---------------------------------------------------------------------------
# qat.py:35-59 decoder: forward values and autograd gradients
# ---------------------------------------------------------------------------
def _fwd_bwd(fn, x, U):
    import torch
    x = torch.from_numpy(x).clone().requires_grad_(True)
    y = fn(x)
    (y * torch.from_numpy(U)).sum().backward()
    return y.detach().numpy(), x.grad.numpy()


@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_fwht_irht_torch(g_qat, dt):
    for n in (1, 2, 8, 32, 256, 512, 4096, 8192):
        k = f"fwht_{dt}_{n}"
        y, gx = _fwd_bwd(O.fwht_torch, g_qat[k + "_x"], g_qat[k + "_U"])
        assert same_bits(y, g_qat[k + "_y"]) and same_bits(gx, g_qat[k + "_gx"]), k
    for n, in0 in ((512, 300), (4096, 4096), (4096, 2999), (16384, 14336)):
        k = f"irht_{dt}_{n}_{in0}"
        if k + "_x" not in g_qat:
            continue
        y, gx = _fwd_bwd(lambda t: O.irht_torch(t, in0), g_qat[k + "_x"], g_qat[k + "_U"])
        assert same_bits(y, g_qat[k + "_y"]) and same_bits(gx, g_qat[k + "_gx"]), k


def recon_exact_grads(states, cw, scg, U, meta, sH, in0):
    """fp64 restatement of the recon_torch gradients: the per-element chain
    in the tensor dtype (as torch's autograd), the two sums exact in fp64."""
    import torch
    n = meta["ncol"]
    g = torch.from_numpy(U) / torch.from_numpy(sH.reshape(1, -1))
    g = torch.nn.functional.pad(g, (0, n - in0))
    g = g * torch.tensor(O.rht_signs(n), dtype=torch.float32)
    g = g / float(np.float32(np.sqrt(n)))
    h = n // 2
    while h >= 1:     # adjoint butterflies, reverse stage order
        v = g.reshape(-1, n // (2 * h), 2, h)
        g = torch.cat([v[:, :, 0, :] + v[:, :, 1, :], v[:, :, 0, :] - v[:, :, 1, :]], dim=2).reshape(-1, n)
        h //= 2
    grec = g.reshape(-1).numpy()
    st = np.asarray(states).reshape(-1)[: grec.size].astype(np.int64)
    grp = np.arange(grec.size) // meta["scale_group"]
    sc = np.asarray(scg, np.float32).reshape(-1)
    t_cw = (grec * sc[grp]).astype(np.float32).astype(np.float64)
    t_sc = (grec * cw[st]).astype(np.float32).astype(np.float64)
    gcw = np.zeros(cw.size)
    np.add.at(gcw, st, t_cw)
    gsc = np.zeros(sc.size)
    np.add.at(gsc, grp, t_sc)
    return gcw, gsc


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_recon_torch(g_qat, tag):
    import torch
    from conftest import grad_close, qat_meta
    k = f"recon_{tag}"
    meta, L, in0 = qat_meta(g_qat, k)
    cw = torch.tensor(O.codebook(L), requires_grad=True)
    scg = torch.tensor(g_qat[k + "_scg"], requires_grad=True)
    Wh = O.recon_torch(g_qat[k + "_states"], cw, scg, meta, torch.from_numpy(g_qat[k + "_sH"]), in0)
    assert same_bits(Wh.detach().numpy(), g_qat[k + "_What"])
    (Wh * torch.from_numpy(g_qat[k + "_U"])).sum().backward()
    assert same_bits(cw.grad.numpy(), g_qat[k + "_gcw"]) and same_bits(scg.grad.numpy(), g_qat[k + "_gsc"])
    # the adjoint chain restated in fp64 sums agrees with torch's fp32 sums
    gcw, gsc = recon_exact_grads(g_qat[k + "_states"], O.codebook(L), g_qat[k + "_scg"], g_qat[k + "_U"],
                                 meta, g_qat[k + "_sH"], in0)
    assert grad_close(gcw.astype(np.float32), g_qat[k + "_gcw"], gcw)
    assert grad_close(gsc.astype(np.float32), g_qat[k + "_gsc"].reshape(-1), gsc)


@pytest.mark.parametrize("L,R,seg", [(8, 2, 64), (12, 2, 64), (10, 3, 256), (16, 4, 256)])
def test_packed_states_roundtrip(g_trellis, L, R, seg):
    """Reference encoder paths are shift-register paths: packing keeps them
    whole in L + R (T-1) bits per sequence."""
    rng = np.random.RandomState(L * 10 + R)
    A = rng.normal(size=(4, 256)).astype(np.float32)
    st, _, _, _ = O.trellis_encode(A, L=L, R=R, seg=seg, scale_group=256)
    pk = O.pack_states(st, L, R)
    assert pk.shape[1] == (L + R * (seg - 1) + 31) // 32
    assert np.array_equal(O.unpack_states(pk, seg, L, R), st)


@pytest.mark.parametrize("tag", ["f32", "f64"])
def test_q8_codec(g_q8, tag):
    """buildq.enc_q8 / qlab.deq_q8 restated: bytes and values bit-exact."""
    q = O.enc_q8(g_q8[f"q8_{tag}_W"])
    assert np.array_equal(q, g_q8[f"q8_{tag}_enc"])
    assert same_bits(O.deq_q8(q), g_q8[f"q8_{tag}_dec"])


def test_block28_transform_restatement():
    """Opt-in H_28 (x) H_P transform: H_28 is a Hadamard matrix, the
    transform is orthogonal and the inverse restores the input."""
    H = O.hadamard28()
    assert np.array_equal(H @ H.T, 28 * np.eye(28, dtype=np.int64))
    rng = np.random.RandomState(28)
    for n0 in (14336, 28672):
        A = rng.normal(size=(2, n0))
        X = O.rht28_rows(A)
        assert abs(np.sum(X ** 2) / np.sum(A ** 2) - 1) < 1e-12
        assert np.abs(O.irht28_rows(X) - A).max() < 1e-13


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_q_uniform(g_quniform, tag):
    A = g_quniform[f"qu_{tag}_A"]
    for bpw in (2, 3, 4, 2.5):
        with np.errstate(invalid="ignore"):
            assert same_bits(O.q_uniform(A, bpw), g_quniform[f"qu_{tag}_{bpw}"])
    assert same_bits(O.q_uniform(A, 3, bs=64), g_quniform[f"qu_{tag}_bs64"])


# ---- finite-codebook E8 (qlab.py:110-124, 185-198) ------------------------------
QE8_CASES = [("qe_A", "qe_A_1.0", 1.0, 256, False), ("qe_A", "qe_A_1.5", 1.5, 256, False),
             ("qe_A", "qe_A_2.0", 2.0, 256, False), ("qe_A", "qe_A32_2.0", 2.0, 256, True),
             ("qe_R", "qe_R_2.0", 2.0, 256, False), ("qe_E", "qe_E_2.0", 2.0, 256, False)]


def _qe8_input(g, key, f32):
    A = g[key]
    return A.astype(np.float32) if f32 else A


def test_e8_codebook_oracle(g_qe8):
    """The oracle's codebook construction reproduces the reference's bytes."""
    import hashlib
    for K, digest in zip(g_qe8["cb_K"], g_qe8["cb_sha256"]):
        assert hashlib.sha256(O.e8_codebook(int(K)).tobytes()).hexdigest() == str(digest)
    assert same_bits(O.e8_codebook(256), g_qe8["cb_256"])


def test_e8_codebook_host(g_qe8):
    """The product's host-side codebook table (numpy, no device) is the
    reference's, bit for bit, for every golden K."""
    import hashlib
    from ultraquant_b200 import qlab as Q
    for K, digest in zip(g_qe8["cb_K"], g_qe8["cb_sha256"]):
        assert hashlib.sha256(Q.e8_codebook(int(K)).tobytes()).hexdigest() == str(digest)


@pytest.mark.parametrize("case", QE8_CASES, ids=[c[1] for c in QE8_CASES])
def test_q_e8_oracle(g_qe8, case):
    key, out, bpw, group, f32 = case
    A = _qe8_input(g_qe8, key, f32)
    # exact distance ties (the edge rows' lone outlier) may pick another codeword
    assert qe8_same_or_tie(O.q_e8(A, bpw, group), g_qe8[out], A, bpw, group) >= 0


def test_q_e8_oracle_group64(g_qe8):
    A = g_qe8["qe_A"][:8]
    assert qe8_same_or_tie(O.q_e8(A, 2.0, group_scale=64), g_qe8["qe_A_g64_2.0"], A, 2.0, 64) == 0


def test_e8_scale_search_restatement():
    """The opt-in per-row scale search (no reference counterpart): every row
    is the reference's q_e8_fast at its chosen step (pinned by the goldens
    above), the total rate does not exceed the global step's, the choice is
    the argmin at the returned lam, and any smaller lam breaks the rate."""
    rng = np.random.RandomState(11)
    A = O.rht_rows(rng.standard_t(4, size=(24, 1024)) / np.sqrt(2) * 0.015)
    step = 0.48
    rec, choice, lam = O.e8_scale_search(A, step)
    D, H = O.e8_scale_search_tables(A, step)
    steps = step * np.array(O.E8_SEARCH_FACTORS)
    for r in range(A.shape[0]):
        assert same_bits(rec[r], O.q_e8_fast(A[r:r + 1], fixed_step=steps[choice[r]]).ravel())
    rows = np.arange(A.shape[0])
    assert H[rows, choice].sum() <= H[:, 8].sum() * (1 + 1e-15)
    assert np.array_equal(choice, np.argmin(D + lam * H, axis=1))
    if lam > 0:
        lower = np.argmin(D + (lam * (1 - 1e-9)) * H, axis=1)
        assert np.cumsum(H[rows, lower])[-1] >= np.cumsum(H[rows, choice])[-1]


@pytest.mark.parametrize("L,R,T", [(6, 1, 32), (6, 3, 32), (8, 2, 64), (8, 4, 64), (12, 2, 64)])
def test_near_tie_codebook_separates_rounding_modes(L, R, T):
    """On the near-tie codebook the reference's two roundings (sub, square,
    add) and a fused multiply-add give different paths on many sequences,
    so a device test on it detects contraction; the C restatement keeps the
    two roundings, like the torch restatement of trellis.py."""
    from conftest import near_tie_codebook
    from oracle import cviterbi as CV
    cb = near_tie_codebook(L, L * 10 + R)
    x = np.random.RandomState(L + R).randn(400, T).astype(np.float32)
    sep = CV.viterbi_segments_c(x, L, R, cw=cb)
    fused = CV.viterbi_segments_c(x, L, R, cw=cb, fused=True)
    assert (sep != fused).any(1).sum() >= 2
    assert np.array_equal(sep[:40], O.viterbi_segments(x[:40], L, R, cb))
