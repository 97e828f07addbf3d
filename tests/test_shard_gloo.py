"""Host-side multi-GPU logic on CPU: the sharding plan, and the exchange steps
(per-tensor error all-gather, row-block assembly) on world_size-2 gloo ranks.
The per-shard quantizer here is the CPU oracle (the device pipelines are
covered by the GPU tests); failures are injected on the host."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
from ultraquant_b200 import shard as S


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_row_once_and_balances(world):
    specs = S.llama_shapes(layers=32)
    shards = S.plan(specs, world)
    cover = {}
    for sh in shards:
        cover.setdefault(sh.tensor.name, []).append((sh.row0, sh.row1))
    for spec in specs:
        spans = sorted(cover[spec.name])
        assert spans[0][0] == 0 and spans[-1][1] == spec.rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    load = [0.0] * world
    for sh in shards:
        load[sh.rank] += sh.tensor.cost(sh.rows)
    assert max(load) / min(load) < 1.01
    # deterministic
    assert [(s.tensor.name, s.row0, s.rank) for s in S.plan(specs, world)] == \
           [(s.tensor.name, s.row0, s.rank) for s in shards]


def test_llama_shapes_match_the_model():
    specs = S.llama_shapes(layers=32)
    assert len(specs) == 224
    total = sum(s.rows * s.cols for s in specs)
    assert total == 32 * (2 * 4096 * 4096 + 2 * 1024 * 4096 + 3 * 14336 * 4096)   # 6.98e9 weights
    padded = sum(s.rows * s.padded_cols for s in specs)
    assert padded > total and padded == total + 32 * 4096 * (16384 - 14336)


SPECS = [S.TensorSpec("t0", 40, 300, L=8, R=2), S.TensorSpec("t1", 24, 256, L=8, R=2),
         S.TensorSpec("t2", 16, 100, L=8, R=2)]


def _weights(spec, r0, r1):
    rng = np.random.RandomState(sum(map(ord, spec.name)))
    W = rng.standard_t(4, size=(spec.rows, spec.cols)) * 0.02
    H = np.exp(rng.normal(0, 1, size=spec.cols))
    return W[r0:r1], H


def _quantize(spec, W, H):
    """E8 recipe on the CPU oracle: returns What and the error sums."""
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = W * sH
    Ah = O.irht_rows(O.q_e8_fast(O.rht_rows(A), fixed_step=0.48), W.shape[1])
    err = torch.tensor([np.sum((A - Ah) ** 2), np.sum(A ** 2)], dtype=torch.float64)
    return torch.from_numpy((Ah / sH).astype(np.float32)), err


def _single_process_reference():
    shards = S.plan(SPECS, 1, block_rows=8)
    res = S.run_shards(shards, 0, _weights, _quantize)
    return S.gather_errors(res, SPECS), {s.name: S.assemble_rows(res, s) for s in SPECS}


def _worker(rank, world, port, out_dir, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        shards = S.plan(SPECS, world, block_rows=8)
        if mode == "rank1_dies" and rank == 1:
            os._exit(3)               # leaves between steps, nothing in flight
        res = S.run_shards(shards, rank, _weights, _quantize)
        errs = S.gather_errors(res, SPECS)
        full = {s.name: S.assemble_rows(res, s, dst_rank=0) for s in SPECS}
        if rank == 0:
            torch.save({"errs": errs, "full": full}, os.path.join(out_dir, "r0.pt"))
    except Exception as e:  # recorded for the failure-detection test
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(type(e).__name__ + ": " + str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_gloo_two_ranks_match_single_process(tmp_path):
    ref_errs, ref_full = _single_process_reference()
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), "ok"), nprocs=2, join=True,
                       start_method="spawn")
    got = torch.load(tmp_path / "r0.pt")
    for name, v in ref_errs.items():
        assert abs(got["errs"][name] - v) <= 1e-12 * v
    for name, t in ref_full.items():
        assert torch.equal(got["full"][name], t)


def test_gloo_rank_failure_is_reported(tmp_path):
    """A rank that exits between steps: the survivor's next collective ends
    with an error within the process-group timeout instead of hanging."""
    import multiprocessing
    ctx = multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), "rank1_dies")) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "survivor did not notice the failed rank"
    assert procs[1].exitcode == 3
    err = (tmp_path / "err0.txt").read_text() if (tmp_path / "err0.txt").exists() else ""
    assert err, "rank 0 should have seen a collective failure"


# ---- calibrated E8 step of a row-sharded tensor (qlab.py:171-180) -------------
CAL_SPEC = S.TensorSpec("cal", 48, 512)


def _cal_blocks(rank, world):
    rng = np.random.RandomState(9)
    W = rng.standard_t(4, size=(CAL_SPEC.rows, CAL_SPEC.cols)) * 0.02
    cut = [0, 16, 40, 48]
    mine = [(0, 3)] if world == 1 else ([(0, 1)] if rank == 0 else [(1, 2), (2, 3)])
    return W, [(cut[a], torch.from_numpy(W[cut[a]:cut[b]])) for a, b in mine]


def _oracle_gn(A, ids):
    return torch.from_numpy(O.group_gn(A.numpy())[ids.numpy()])


def _cal_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        _, blocks = _cal_blocks(rank, world)
        step = S.calibrate_e8(blocks, CAL_SPEC, 1.0, sample_gn=_oracle_gn,
                              bisect=lambda sub: O.e8_bisect(sub.numpy(), 1.0))
        torch.save(step, os.path.join(out_dir, f"step{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gloo_sharded_e8_calibration_matches_single_process(tmp_path):
    """Two ranks holding uneven row blocks (rank 1 two of them) draw the same
    sample, gather the normalised vectors and get the single-process step."""
    W, _ = _cal_blocks(0, 1)
    cache = {}
    O.q_e8_fast(W, 1.0, calib_key="k", cache=cache)
    assert 0.31 < cache["k"] < 9.9            # an interior step, not a bracket end
    mp.start_processes(_cal_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        assert torch.load(tmp_path / f"step{r}.pt") == cache["k"]


# ---- packed trellis codes of row-sharded tensors (qat.py:11-33 codes) ---------
CODE_SPECS = [S.TensorSpec("c0", 24, 256, L=8, R=2), S.TensorSpec("c1", 16, 300, L=8, R=3),
              S.TensorSpec("c2", 8, 512, L=6, R=1)]
SEG, GROUP = 64, 256


def _oracle_codes(spec, W, H):
    """Oracle trellis recipe on a block of rows: packed codes, scales, error sums."""
    Hc = np.maximum(H, H.max() * 1e-3)
    sH = np.sqrt(Hc)[None, :]
    A = W * sH
    Ar = O.rht_rows(A)
    st, sc_g, cw, meta = O.trellis_encode(Ar, L=spec.L, R=spec.R, seg=SEG, scale_group=GROUP)
    Ah = O.irht_rows(O.trellis_decode(st, cw, sc_g, meta), W.shape[1])
    err = torch.tensor([np.sum((A - Ah) ** 2), np.sum(A ** 2)], dtype=torch.float64)
    codes = torch.from_numpy(O.pack_states(st, spec.L, spec.R).view(np.int32))
    return st, codes, torch.from_numpy(sc_g.reshape(-1).astype(np.float32)), err


def _codes_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        shards = S.plan(CODE_SPECS, world, block_rows=8)
        local = []
        for s in shards:
            if s.rank == rank:
                W, H = _weights(s.tensor, s.row0, s.row1)
                _, codes, sc, err = _oracle_codes(s.tensor, W, H)
                local.append(S.ShardCodes(s, codes, sc, err))
        out = S.gather_codes(local, shards, world, seg=SEG, group=GROUP)
        torch.save({k: (v.codes, v.sc, v.err) for k, v in out.items()}, os.path.join(out_dir, f"codes{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gloo_gathered_codes_unpack_to_single_process_states(tmp_path):
    """Two ranks quantize interleaved row blocks of three tensors; after the
    one all-gather, both ranks hold packed codes that unpack to the states of
    the whole tensor quantized in one process, with its scales, and the
    block error sums add up to its weighted NMSE."""
    mp.start_processes(_codes_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    shards = S.plan(CODE_SPECS, 2, block_rows=8)
    assert {s.rank for s in shards} == {0, 1}
    for r in range(2):
        got = torch.load(tmp_path / f"codes{r}.pt")
        for spec in CODE_SPECS:
            W, H = _weights(spec, 0, spec.rows)
            st, codes, sc, err = _oracle_codes(spec, W, H)
            gc, gsc, gerr = got[spec.name]
            assert torch.equal(gc, codes), spec.name
            assert np.array_equal(O.unpack_states(gc.numpy().view(np.uint32), SEG, spec.L, spec.R), st)
            assert torch.equal(gsc.view(torch.int32), sc.view(torch.int32))
            assert abs(float(gerr[0] / gerr[1]) - float(err[0] / err[1])) <= 1e-12 * float(err[0] / err[1])


# ---- resumable runs: per-row-block completion markers (BlockStore) -------------

def test_block_store_round_trip_and_markers(tmp_path):
    """Saved blocks load back bit-identically; a block counts as done only
    with its marker, for the same L, R, seg and group, and a file that does
    not match the block's plan is not used."""
    shards = S.plan(CODE_SPECS, 1, block_rows=8)
    store = S.BlockStore(str(tmp_path), rank=0)
    saved = {}
    for s in shards[:-1]:
        W, H = _weights(s.tensor, s.row0, s.row1)
        _, codes, sc, err = _oracle_codes(s.tensor, W, H)
        c = S.ShardCodes(s, codes, sc, err)
        store.save(c, SEG, GROUP)
        saved[(s.tensor.name, s.row0)] = c
    fresh = S.BlockStore(str(tmp_path), rank=1)          # another process, another rank
    for s in shards[:-1]:
        assert fresh.done(s, SEG, GROUP)
        assert not fresh.done(s, SEG * 2, GROUP)          # other parameters: not this block
        got = fresh.load(s, "cpu", SEG, GROUP)
        ref = saved[(s.tensor.name, s.row0)]
        assert torch.equal(got.codes, ref.codes) and torch.equal(got.sc.view(torch.int32), ref.sc.view(torch.int32))
        assert torch.equal(got.err, ref.err)
    last = shards[-1]
    assert not fresh.done(last, SEG, GROUP)
    # a block file written without its marker (interrupted before the marker) is not done
    W, H = _weights(last.tensor, last.row0, last.row1)
    _, codes, sc, err = _oracle_codes(last.tensor, W, H)
    np.savez(store.path(last), codes=codes.numpy(), sc=sc.numpy(), err=err.numpy())
    assert not S.BlockStore(str(tmp_path)).done(last, SEG, GROUP)
    # a marked block whose file does not match its plan is not loaded
    first = shards[0]
    np.savez(store.path(first), codes=codes.numpy()[:1], sc=sc.numpy(), err=err.numpy())
    assert S.BlockStore(str(tmp_path)).load(first, "cpu", SEG, GROUP) is None


def _store_worker(rank, world, port, root):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        store = S.BlockStore(root, rank=rank)
        for s in S.plan(CODE_SPECS, world, block_rows=8):
            if s.rank == rank:
                W, H = _weights(s.tensor, s.row0, s.row1)
                _, codes, sc, err = _oracle_codes(s.tensor, W, H)
                store.save(S.ShardCodes(s, codes, sc, err), SEG, GROUP)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_resume_at_another_world_size(tmp_path):
    """Two gloo ranks quantize and save their row blocks; a re-run in one
    process takes every block from the store (no block is quantized again:
    its weight callback raises) and gathers the codes of the whole tensors
    quantized in one process."""
    root = str(tmp_path / "store")
    mp.start_processes(_store_worker, args=(2, _free_port(), root), nprocs=2, join=True, start_method="spawn")
    assert sorted(f for f in os.listdir(root) if f.endswith(".done")) == ["blocks.0.done", "blocks.1.done"]

    def no_weights(s):
        raise AssertionError(f"block {s.tensor.name}:{s.row0} quantized again")

    shards = S.plan(CODE_SPECS, 1, block_rows=8)
    local = S.quantize_shards(shards, 0, no_weights, seg=SEG, group=GROUP, store=S.BlockStore(root), device="cpu")
    assert len(local) == len(shards)
    out = S.gather_codes(local, shards, 1, seg=SEG, group=GROUP)
    for spec in CODE_SPECS:
        W, H = _weights(spec, 0, spec.rows)
        st, codes, sc, err = _oracle_codes(spec, W, H)
        assert torch.equal(out[spec.name].codes, codes), spec.name
        assert torch.equal(out[spec.name].sc.view(torch.int32), sc.view(torch.int32))
        assert abs(out[spec.name].wnmse - float(err[0] / err[1])) <= 1e-12 * float(err[0] / err[1])


# ---- int16 E8 points of row-sharded tensors (qlab.py:153, 159-183) -------------
E8_SPECS = [S.TensorSpec("e0", 24, 256), S.TensorSpec("e1", 16, 300), S.TensorSpec("e2", 8, 512)]
E8_STEP = 0.48


def _oracle_e8(spec, W, H):
    """Oracle fixed-step E8 recipe on a block of rows: int16 points 2p of the
    padded rotated rows and the error sums."""
    Hc = np.maximum(H, H.max() * 1e-3)
    A = W * np.sqrt(Hc)[None, :]
    Ar = O.rht_rows(A)
    p = O.e8_decode(O.group_gn(Ar) / E8_STEP)
    idx = torch.from_numpy((2 * p).reshape(Ar.shape).astype(np.int16))
    Ah = O.irht_rows(O.q_e8_fast(Ar, fixed_step=E8_STEP), W.shape[1])
    err = torch.tensor([np.sum((A - Ah) ** 2), np.sum(A ** 2)], dtype=torch.float64)
    return idx, err


def _e8_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        shards = S.plan(E8_SPECS, world, block_rows=8)
        local = []
        for s in shards:
            if s.rank == rank:
                W, H = _weights(s.tensor, s.row0, s.row1)
                idx, err = _oracle_e8(s.tensor, W, H)
                local.append(S.ShardE8(s, idx, err))
        out = S.gather_e8(local, shards, world, E8_STEP)
        torch.save({k: (v.idx, v.err) for k, v in out.items()}, os.path.join(out_dir, f"e8_{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gloo_gathered_e8_points_equal_single_process(tmp_path):
    """Two ranks quantize interleaved row blocks with the fixed-step E8
    recipe; after the one all-gather both hold the int16 points of the whole
    tensors quantized in one process and their weighted NMSE."""
    mp.start_processes(_e8_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert {s.rank for s in S.plan(E8_SPECS, 2, block_rows=8)} == {0, 1}
    for r in range(2):
        got = torch.load(tmp_path / f"e8_{r}.pt")
        for spec in E8_SPECS:
            W, H = _weights(spec, 0, spec.rows)
            idx, err = _oracle_e8(spec, W, H)
            gidx, gerr = got[spec.name]
            assert gidx.shape == (spec.rows, spec.padded_cols)
            assert torch.equal(gidx, idx), spec.name
            assert abs(float(gerr[0] / gerr[1]) - float(err[0] / err[1])) <= 1e-12 * float(err[0] / err[1])


def _idle_rank_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        spec = CODE_SPECS[2]                               # 8 rows: one block, on rank 0
        shards = S.plan([spec], world, block_rows=8)
        local = []
        for s in shards:
            if s.rank == rank:
                W, H = _weights(s.tensor, s.row0, s.row1)
                _, codes, sc, err = _oracle_codes(s.tensor, W, H)
                local.append(S.ShardCodes(s, codes, sc, err))
        out = S.gather_codes(local, shards, world, seg=SEG, group=GROUP)
        torch.save((len(local), out[spec.name].codes), os.path.join(out_dir, f"idle{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gather_with_a_rank_without_blocks(tmp_path):
    """More ranks than blocks: the idle rank still takes part in the one
    all-gather and receives the whole tensor's codes."""
    mp.start_processes(_idle_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    spec = CODE_SPECS[2]
    W, H = _weights(spec, 0, spec.rows)
    _, codes, _, _ = _oracle_codes(spec, W, H)
    n0, c0 = torch.load(tmp_path / "idle0.pt")
    n1, c1 = torch.load(tmp_path / "idle1.pt")
    assert (n0, n1) == (1, 0)
    assert torch.equal(c0, codes) and torch.equal(c1, codes)
