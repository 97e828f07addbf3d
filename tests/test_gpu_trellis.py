"""GPU parity: codebook, Viterbi encoder / decoder and the fused pipelines
against the reference goldens and the oracle, through the C ABI."""
import numpy as np
import pytest

import oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu

TQ = ["l8r2", "l8r1", "l8r3", "l8r4", "l10r2", "l12r2", "l12r2s64", "l12r3", "l16r2", "l16r3", "pad", "g128"]


@pytest.fixture(scope="module")
def T():
    import ultraquant_b200.trellis as T
    return T


@pytest.fixture(scope="module")
def Qat():
    import ultraquant_b200.qat as Qat
    return Qat


def test_codebook_exhaustive(T, g_trellis):
    """All 2^16 states (smaller L are prefixes) equal scipy's norm.ppf table."""
    cb = T.codebook(16)
    ref = g_trellis["codebook16"]
    bad = np.nonzero(cb.view(np.int32) != ref.view(np.int32))[0]
    assert bad.size == 0, f"{bad.size} codewords differ, first {bad[:5]}"
    assert same_bits(T.codebook(12), ref[:4096])


@pytest.mark.parametrize("tag", TQ)
def test_trellis_golden(T, Qat, g_trellis, tag):
    A = g_trellis[f"tq_{tag}_in"]
    L, R, seg, group = (int(v) for v in g_trellis[f"tq_{tag}_cfg"])
    rec = T.trellis_quant_fast(A, L=L, R=R, seg=seg, scale_group=group)
    assert same_bits(rec, g_trellis[f"tq_{tag}_rec"])
    st, sc_g, cw, meta = Qat.trellis_encode(A, L=L, R=R, seg=seg, scale_group=group)
    assert np.array_equal(st, g_trellis[f"tq_{tag}_states"])
    assert same_bits(sc_g, g_trellis[f"tq_{tag}_scg"])


@pytest.mark.parametrize("tag", ["r8", "r10"])
def test_trellis_full_row_golden(T, g_trellis, tag):
    A = g_trellis[f"tr_{tag}_in"]
    L, R, group = (int(v) for v in g_trellis[f"tr_{tag}_cfg"])
    assert same_bits(T.trellis_quant(A, L=L, R=R, group=group), g_trellis[f"tr_{tag}_rec"])


@pytest.mark.parametrize("L,R,seg", [(6, 1, 32), (6, 2, 64), (6, 3, 16), (8, 4, 64), (9, 2, 64), (10, 1, 256),
                                     (11, 3, 256), (12, 2, 256), (13, 2, 128), (14, 2, 256), (14, 4, 256),
                                     (15, 2, 64), (15, 3, 256), (16, 1, 256), (16, 2, 256), (16, 3, 256),
                                     (16, 4, 256), (12, 2, 1), (12, 2, 2), (16, 2, 1)])
def test_viterbi_states_vs_oracle(T, L, R, seg):
    """Random sequences (plus exact-valued ones that provoke cost ties)."""
    import torch
    rng = np.random.RandomState(L * 100 + R * 10 + seg)
    nseq = 24 if L >= 15 else 70
    x = rng.randn(nseq, seg).astype(np.float32)
    x[:4] = np.round(x[:4] * 2) / 2
    got = T.viterbi_states(torch.from_numpy(x).cuda(), L, R).cpu().numpy()
    ref = O.viterbi_segments(x, L, R)
    assert np.array_equal(got, ref)


def test_trellis_fast_full_size_l12(T, Qat):
    """Config-1 shape: 4096 x 4096, L=12 R=2, T=256 (65,536 sequences).
    Size-independent checks on all of it, bit-exact oracle on a subsample."""
    import torch
    rng = np.random.RandomState(0)
    W = rng.normal(0, 0.02, size=(4096, 4096))
    m = rng.random_sample(W.shape) < 0.001
    W[m] = np.sign(rng.normal(size=m.sum())) * 0.16
    A = torch.from_numpy(W.astype(np.float32)).cuda()
    st, sc, ntot, pad = T.encode_segments(A, 12, 2, 256, 256)
    assert st.shape == (65536, 256) and int(st.min()) >= 0 and int(st.max()) < 4096
    # bitshift structure: s_t >> R == s_{t-1} & (2^(L-R) - 1)
    assert bool(((st[:, 1:] >> 2) == (st[:, :-1] & 1023)).all())
    rec = T.trellis_quant_fast(A, L=12, R=2, seg=256, scale_group=256)
    nmse = float(((rec - A) ** 2).sum() / (A ** 2).sum())
    assert 0.05 < nmse < 0.1, nmse
    pick = np.sort(rng.choice(65536, 48, replace=False))
    xs = (A.reshape(-1, 256)[pick] / sc[pick].reshape(-1, 1)).cpu().numpy()
    ref = O.viterbi_segments(xs, 12, 2)
    assert np.array_equal(st[pick].cpu().numpy(), ref)


def test_pipeline_golden(g_pipeline):
    from ultraquant_b200 import pipeline as P
    W, H = g_pipeline["W"], g_pipeline["H"]
    for L, R, seg in [(8, 2, 64), (12, 2, 64), (10, 3, 256)]:
        res = P.quant_trellis_device(__import__("torch").from_numpy(W).cuda(),
                                     __import__("torch").from_numpy(H).cuda(), L, R, seg, 256)
        assert same_bits(res.What.cpu().numpy(), g_pipeline[f"qt_{L}_{R}_{seg}_What"])
        ref = float(g_pipeline[f"qt_{L}_{R}_{seg}_wnmse"])
        assert abs(res.wnmse - ref) <= 1e-5 * ref
    for step in (0.48, 0.25):
        assert same_bits(P.quant_step(W, H, step), g_pipeline[f"qs_{step}_What"])


def test_pipeline_l16_vs_oracle():
    """Config-2 recipe (L=16, k=2 and k=3, T=256, log-normal imatrix) on a
    slice of rows: What bit-exact, weighted NMSE within 1e-5 relative."""
    import torch
    from ultraquant_b200 import pipeline as P
    rng = np.random.RandomState(1)
    W = rng.normal(0, 0.02, size=(4, 4096)).astype(np.float32)
    H = np.exp(rng.normal(0.0, 1.0, size=4096))
    for R in (2, 3):
        res = P.quant_trellis_device(torch.from_numpy(W).cuda(), torch.from_numpy(H).cuda(), 16, R, 256, 256)
        ref = O.quant_trellis(W.astype(np.float64), H, L=16, R=R, seg=256)
        assert same_bits(res.What.cpu().numpy(), ref)
        Hc = np.maximum(H, H.max() * 1e-3)
        sH = np.sqrt(Hc)[None, :]
        A = W.astype(np.float64) * sH
        Ah = O.irht_rows(O.trellis_quant_fast(O.rht_rows(A), L=16, R=R, seg=256), 4096)
        w = O.wnmse(A, Ah)
        assert abs(res.wnmse - w) <= 1e-5 * w


def test_install_patches_reference_modules(tmp_path, monkeypatch):
    """install() swaps the hot path into importable qlab / trellis / qat
    modules (here: stand-ins with the reference's attribute names)."""
    import sys
    for name, body in {"qlab": "def rht_rows(A, seed=0): raise AssertionError\n_E8_SCALE = {}\n"
                               "def load_WH(n): return n\n",
                       "trellis": "def trellis_quant_fast(*a, **k): raise AssertionError\n",
                       "qat": "DEV='cuda'\n"}.items():
        (tmp_path / f"{name}.py").write_text(body)
    monkeypatch.syspath_prepend(str(tmp_path))
    for name in ("qlab", "trellis", "qat"):
        sys.modules.pop(name, None)
    import ultraquant_b200
    mods = ultraquant_b200.install()
    from qlab import rht_rows, load_WH
    import ultraquant_b200.qlab as Q
    assert rht_rows is Q.rht_rows and load_WH("x") == "x"
    A = np.random.RandomState(0).randn(3, 100)
    assert same_bits(mods["qlab"].rht_rows(A), O.rht_rows(A))
    import ultraquant_b200.qat as Qat
    assert mods["qat"].recon_torch is Qat.recon_torch and mods["qat"].fwht_torch is Qat.fwht_torch
    for name in ("qlab", "trellis", "qat"):
        sys.modules.pop(name, None)


def test_bounded_wait_reports_timeout():
    """The device waits of the cluster exchange are bounded: a wait on a
    barrier phase that nothing completes gives up and the host reads
    UQ_ERR_TIMEOUT; the context stays usable afterwards."""
    import torch
    from ultraquant_b200 import _device as D
    from ultraquant_b200 import _lib
    lib = _lib.load()
    st = D.stream_handle(D.device())
    assert lib.uq_wait_timeout_selftest(50.0, st) == _lib.UQ_ERR_TIMEOUT
    assert lib.uq_device_errors(st) == _lib.UQ_OK
    x = torch.randn(2, 64, device="cuda")
    import ultraquant_b200.trellis as T
    assert T.viterbi_states(x, 12, 2).shape == (2, 64)


@pytest.mark.parametrize("T,L,R", [(256, 16, 2), (256, 16, 3), (64, 12, 2), (256, 10, 3), (33, 8, 1),
                                   (1, 16, 4), (2, 6, 3), (256, 16, 4)])
def test_pack_states_vs_oracle(T, L, R):
    """Packed codes: device words equal the oracle's bit strings for random
    shift-register paths (R = 3 fields straddle words), unpack inverts."""
    import ultraquant_b200.trellis as T_
    rng = np.random.RandomState(T * 100 + L * 10 + R)
    nseq = 37
    st = np.zeros((nseq, T), dtype=np.int32)
    st[:, 0] = rng.randint(0, 1 << L, nseq)
    for t in range(1, T):
        st[:, t] = ((st[:, t - 1].astype(np.int64) << R) | rng.randint(0, 1 << R, nseq)) & ((1 << L) - 1)
    pk = T_.pack_states(st, L, R)
    assert pk.dtype == np.uint32 and np.array_equal(pk, O.pack_states(st, L, R))
    assert np.array_equal(T_.unpack_states(pk, T, L, R), st)


def test_pack_viterbi_paths_roundtrip():
    """Viterbi output (L = 16, R = 2 and 3) survives pack -> unpack on the device;
    (L + R (T-1)) / T bits per weight."""
    import torch
    import ultraquant_b200.trellis as T_
    x = torch.randn(300, 256, device="cuda")
    for R in (2, 3):
        st = T_.viterbi_states(x, 16, R)
        pk = T_.pack_states(st, 16, R)
        assert pk.shape == (300, (16 + R * 255 + 31) // 32)
        assert torch.equal(T_.unpack_states(pk, 256, 16, R), st)


@pytest.mark.parametrize("L,R,nseq,fit", [(12, 2, 3000, 2500), (16, 2, 400, 300), (16, 3, 300, 200)])
def test_viterbi_small_workspace_batches(L, R, nseq, fit):
    """A workspace that holds only `fit` sequences: the entry point runs
    several backpointer batches, each cut down to whole waves of resident
    CTAs (clusters at L = 16), and returns the states of a single batch."""
    import torch
    from ultraquant_b200 import _device as D
    from ultraquant_b200 import _lib
    lib = _lib.load()
    T = 256
    torch.manual_seed(nseq + L)
    x = torch.randn(nseq, T, device="cuda")
    cw = D.codebook(L, x.device)

    def run(ws_bytes):
        out = torch.full((nseq, T), -1, dtype=torch.int32, device=x.device)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        rc = lib.uq_trellis_viterbi(x.data_ptr(), nseq, T, L, R, cw.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                    ws.numel(), D.stream_handle(x.device))
        assert rc == 0, lib.uq_last_error()
        return out

    per_seq = (T - 1) * ((1 << L) // 64) * 4 + 4
    full = run(lib.uq_trellis_workspace_bytes(nseq, T, L, R))
    small = run(fit * per_seq + 512)
    torch.cuda.synchronize()
    assert torch.equal(small, full)
    assert int(full.min()) >= 0 and int(full.max()) < (1 << L)


def test_pipeline_reports_injected_device_timeouts():
    """A bounded device wait that gave up leaves its kernel's outputs wrong;
    the production wrappers must raise instead of returning them.  The flag
    is set on the host (no kernel is made to time out here), and the next
    call after the report runs clean."""
    import torch
    from ultraquant_b200 import _lib, pipeline as P, qlab as Q
    lib = _lib.load()
    rng = np.random.RandomState(3)
    W = torch.from_numpy(rng.normal(0, 0.02, size=(8, 4096)).astype(np.float32)).cuda()
    H = torch.from_numpy(np.exp(rng.normal(0, 1, size=4096))).cuda()
    calls = [lambda: P.quant_trellis_device(W, H, 16, 2, 256, 256),
             lambda: P.quant_step_device(W, H, 0.48),
             lambda: Q.rht_rows(W.double())]
    for which in (0, 1, 2):
        for call in calls:
            assert lib.uq_inject_device_flag(which) == _lib.UQ_OK
            with pytest.raises(_lib.UQError, match="timed out"):
                call()
            call()   # flag cleared by the report
    assert lib.uq_inject_device_flag(7) == _lib.UQ_ERR_INVALID


def test_sharded_codes_match_whole_tensor():
    """shard.quantize_shards + gather_codes over several row blocks (one
    process) give the packed codes, scales and weighted NMSE of the whole
    tensor quantized in one call, and the codes unpack to its states."""
    import torch
    from ultraquant_b200 import pipeline as P, shard as S, trellis as Tr
    rng = np.random.RandomState(5)
    rows, cols = 1536, 4096
    W = torch.from_numpy(rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)).cuda()
    H = torch.from_numpy(np.exp(rng.normal(0, 1, size=cols))).cuda()
    for R in (2, 3):
        spec = S.TensorSpec(f"t{R}", rows, cols, L=16, R=R)
        plan = S.plan([spec], 1, block_rows=512)
        assert len(plan) == 3
        loc = S.quantize_shards(plan, 0, lambda s: (W[s.row0:s.row1], H), 256, 256)
        out = S.gather_codes(loc, plan, 1, 256, 256)[spec.name]
        whole = P.quant_trellis_device(W, H, 16, R, 256, 256)
        assert torch.equal(out.codes, Tr.pack_states(whole.states, 16, R))
        assert torch.equal(Tr.unpack_states(out.codes, 256, 16, R), whole.states)
        assert torch.equal(out.sc.view(torch.int32), whole.sc.view(torch.int32))
        assert abs(out.wnmse - whole.wnmse) <= 1e-12 * whole.wnmse


def test_sharded_e8_points_match_whole_tensor():
    """shard.quantize_shards_e8 + gather_e8 over three row blocks give the
    int16 E8 points and weighted NMSE of the whole tensor quantized in one
    call (ffn_down width 14336 -> 16384, step 0.48)."""
    import torch
    from ultraquant_b200 import pipeline as P, shard as S
    rng = np.random.RandomState(8)
    rows, cols = 1536, 14336
    W = torch.from_numpy((rng.standard_t(4, size=(rows, cols)) / np.sqrt(2) * 0.015).astype(np.float32)).cuda()
    H = torch.from_numpy(np.exp(rng.normal(0, 1, size=cols))).cuda()
    spec = S.TensorSpec("d", rows, cols)
    plan = S.plan([spec], 1, block_rows=512)
    assert len(plan) == 3
    out = S.gather_e8(S.quantize_shards_e8(plan, 0, lambda s: (W[s.row0:s.row1], H), 0.48), plan, 1, 0.48)[spec.name]
    whole = P.quant_step_device(W, H, 0.48, keep_codes=True)
    assert torch.equal(out.idx.reshape(-1), whole.idx)
    assert abs(out.wnmse - whole.wnmse) <= 1e-12 * whole.wnmse


def test_quantize_shards_resumes_from_block_store(tmp_path):
    """A run saves its three row blocks to a BlockStore; a crash that lost the
    second block's marker is simulated by deleting that marker line.  The
    re-run quantizes only that block, loads the others, and gathers the codes,
    scales and weighted NMSE of a run without the store."""
    import torch
    from ultraquant_b200 import shard as S
    rng = np.random.RandomState(6)
    rows, cols = 1536, 4096
    W = torch.from_numpy(rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)).cuda()
    H = torch.from_numpy(np.exp(rng.normal(0, 1, size=cols))).cuda()
    spec = S.TensorSpec("w", rows, cols, L=16, R=2)
    plan = S.plan([spec], 1, block_rows=512)
    ref = S.gather_codes(S.quantize_shards(plan, 0, lambda s: (W[s.row0:s.row1], H)), plan, 1)[spec.name]
    root = str(tmp_path)
    S.quantize_shards(plan, 0, lambda s: (W[s.row0:s.row1], H), store=S.BlockStore(root))
    marker = tmp_path / "blocks.0.done"
    lines = marker.read_text().splitlines()
    assert len(lines) == 3
    lost = S.BlockStore.key(plan[1], 256, 256)
    assert lost in lines
    marker.write_text("\n".join(ln for ln in lines if ln != lost) + "\n")
    called = []

    def weights(s):
        called.append(s.row0)
        return W[s.row0:s.row1], H

    loc = S.quantize_shards(plan, 0, weights, store=S.BlockStore(root))
    assert called == [plan[1].row0]
    out = S.gather_codes(loc, plan, 1)[spec.name]
    assert torch.equal(out.codes, ref.codes)
    assert torch.equal(out.sc.view(torch.int32), ref.sc.view(torch.int32))
    assert out.wnmse == ref.wnmse
    assert len(marker.read_text().splitlines()) == 3


@pytest.mark.parametrize("L,R,T,n", [(6, 1, 32, 2000), (6, 3, 32, 2000), (8, 2, 64, 2000), (8, 4, 64, 2000),
                                     (12, 2, 64, 2000), (12, 3, 64, 2000), (14, 2, 64, 400), (15, 3, 64, 400),
                                     (16, 1, 32, 64), (16, 2, 32, 128), (16, 3, 32, 128), (16, 4, 32, 64)])
def test_viterbi_two_roundings_on_near_ties(T, L, R, n):
    """Every cost is RN(RN((x - cw)^2) + m) like trellis.py's separate torch
    ops, never a fused multiply-add: on the near-tie codebook (entries a few
    ulps apart) contraction changes the path on many sequences, and the
    device must return the separately rounded oracle's states on all."""
    import torch
    from conftest import near_tie_codebook
    from oracle import cviterbi as CV
    cb = near_tie_codebook(L, L * 10 + R)
    x = np.random.RandomState(L + R + T).randn(n, T).astype(np.float32)
    ref = CV.viterbi_segments_c(x, L, R, cw=cb)
    fused = CV.viterbi_segments_c(x, L, R, cw=cb, fused=True)
    assert (ref != fused).any(1).sum() >= 1, "the case does not separate the rounding modes"
    got = T_viterbi(torch.from_numpy(x).cuda(), L, R, torch.from_numpy(cb).cuda())
    bad = np.flatnonzero((got != ref).any(1))
    assert bad.size == 0, f"{bad.size} of {n} sequences differ from the two-rounding oracle (first {bad[:5]})"


def T_viterbi(x, L, R, cw):
    import ultraquant_b200.trellis as Tr
    return Tr.viterbi_states(x, L, R, cw).cpu().numpy()


def test_bench_tensor_sequence_with_one_ulp_best_paths():
    """The one sequence of the benchmarked tensor (seed 0, row 30, segment 7,
    L = 16, k = 3) whose two best final costs are one fp32 ulp apart: a
    contracted multiply-add picked the second."""
    import torch
    import bench
    from oracle.uq_oracle import _flat_normalise
    from oracle import cviterbi as CV
    W, H = bench.make_inputs(0)
    Hc = np.maximum(H, H.max() * 1e-3)
    A = W[30:31].astype(np.float64) * np.sqrt(Hc)[None, :]
    xn, _, _, _ = _flat_normalise(O.rht_rows(A), 256, 256)
    x = np.ascontiguousarray(xn[7:8])
    ref = CV.viterbi_segments_c(x, 16, 3)
    assert not np.array_equal(ref, CV.viterbi_segments_c(x, 16, 3, fused=True))
    import ultraquant_b200.trellis as Tr
    assert np.array_equal(Tr.viterbi_states(torch.from_numpy(x).cuda(), 16, 3).cpu().numpy(), ref)
