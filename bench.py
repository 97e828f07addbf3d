#!/usr/bin/env python
"""Benchmark: trellis-quantized weights/s on B200.

Workload (the configuration the metric is quoted on): one 4096 x 4096 float32
weight matrix, N(0, 0.02^2) from seed 0 with 0.1 % of the entries replaced by
+-8 sigma outliers, and a log-normal(0, 1) per-column imatrix.  One step runs
the importance-weighted trellis recipe of buildtrellis.py -- A = W*sqrt(H),
RHT (fp64), per-256 RMS, Viterbi with L = 16 state bits and T = 256, decode,
inverse RHT, /sqrt(H), weighted-error statistics -- at k = 3 and at k = 2
bits/weight, packs every sequence's state path into its L + R(T-1) bits, and
ends with every rank holding the whole tensor's packed codes, per-256 scales
and per-tensor error sums.  Synthetic, seeded inputs stand in for real
checkpoints.

Multi-GPU (torchrun, one process per GPU): the same tensor is split by row
blocks across the ranks ("strong" scaling: the work per step is fixed); each
rank quantizes its rows and the step ends with ONE NCCL all-gather of the
packed codes, scales and error sums (the path's only exchange).  Time = max
over ranks of the CUDA-event time; value = the tensor's weights (both k) per
second.

value     : weights quantized per second, inputs resident in HBM.
e2e       : the same through the public API (ultraquant_b200.shard) with the
            rank's rows in pinned host memory: host->device copies, the
            quantization, the gather, and device->host copies of What and (rank
            0) the gathered codes are all inside the timed region.
roofline  : the Viterbi forward kernel (the step's dominant kernel) against a
            MEASURED FP32 lane peak (uq_fp32_lane_probe, same process);
            roofline_kernels: the RHT and E8 kernels against measured HBM.
cpu_baseline / --impl reference : the CPU restatement of the reference's
            torch path (oracle/) on the host cores, on a bounded row sample.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "trellis-quantized weights/sec (L=16, T=256, k=2 and k=3, importance-weighted RHT pipeline)"
UNIT = "weights/s"
ROWS = COLS = 4096
L_BITS = 16
KS = (3, 2)
SEG = 256
GROUP = 256
HBM_FALLBACK_GBS = 6650.0

# ncu (L=16, T=256, one launch of 296 sequences per k): DRAM read + write
# bytes of viterbi_fwd_kernel per sequence (the traffic is the backpointers)
NCU_DRAM_BYTES_PER_SEQ = {2: (0.899072e6 + 559.365888e6) / 296, 3: (0.901888e6 + 561.186304e6) / 296}


def make_inputs(seed: int):
    import numpy as np
    rng = np.random.RandomState(seed)
    W = rng.normal(0.0, 0.02, size=(ROWS, COLS))
    m = rng.random_sample(W.shape) < 0.001
    W[m] = np.sign(rng.normal(size=int(m.sum()))) * 8 * 0.02
    H = np.exp(rng.normal(0.0, 1.0, size=COLS))
    return W.astype(np.float32), H


def ops_per_weight(L: int, R: int) -> int:
    """Algorithmic lane ops of one Viterbi step per weight: sub, mul, add per
    state plus (2^R - 1) compares per predecessor group."""
    return 3 * (1 << L) + ((1 << R) - 1) * (1 << (L - R))


def measured_peaks():
    """HBM GB/s from the pool's MEASURED_PEAKS.json, else the fallback figure."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, ValueError, KeyError, TypeError):
        return HBM_FALLBACK_GBS, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def host_info():
    import numpy as np
    import torch
    model = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        affinity = len(os.sched_getaffinity(0))
    except AttributeError:
        affinity = os.cpu_count()
    info = {"host_cpus": os.cpu_count(), "cpus_usable": affinity, "cpu_model": model,
            "numpy": np.__version__, "torch": torch.__version__}
    try:
        import scipy
        info["scipy"] = scipy.__version__
    except ImportError:
        pass
    return info


class ClockSampler:
    """nvidia-smi clock / throttle samples (every 200 ms).  Started before
    the warm-up, so that nvidia-smi's start-up does not fall into the timed
    region; mark() brackets the timed region and summary() keeps only the
    samples taken inside it."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None
        self.t0 = self.t1 = None

    def mark(self, start: bool):
        if start:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.f is None:
            return None
        try:
            rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
            os.unlink(self.f.name)
        except Exception:
            return None
        import datetime
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        def stamp(r):
            try:
                return datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except (ValueError, IndexError):
                return None
        stamped = self.t0 is not None and any(stamp(r) is not None for r in rows)
        for r in rows:
            ts = stamp(r)
            r = [x.strip() for x in r]
            # samples inside the timed region (a quarter period of slack)
            if stamped and (ts is None or not (self.t0 - 0.05 <= ts <= (self.t1 or ts) + 0.05)):
                continue
            try:
                sm.append(float(r[2]))
                mx.append(float(r[3]))
                pw.append(float(r[4]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, r[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(pw) if pw else None}


def phys_gpu_index(local: int) -> int:
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [p.strip() for p in phys.split(",")] if phys else []
    return int(parts[local]) if local < len(parts) and parts[local].isdigit() else local


# ---------------------------------------------------------------------------
# CPU legs (reference arm, cpu_baseline)
# ---------------------------------------------------------------------------
def use_all_host_threads() -> int:
    """torch.distributed.run sets OMP_NUM_THREADS=1 for every rank; the CPU
    legs run on rank 0 alone, so give torch every core this process may use."""
    import torch
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(max(1, n))
    return torch.get_num_threads()


def cpu_reference_sample(W, H, rows: int):
    """Oracle restatement of the reference path on `rows` rows (k=3 and k=2)."""
    import numpy as np
    import torch
    import oracle as O
    Wd = W[:rows].astype(np.float64)
    t0 = time.perf_counter()
    for R in KS:
        O.quant_trellis(Wd, H, L=L_BITS, R=R, seg=SEG, scale_group=GROUP)
    dt = time.perf_counter() - t0
    return rows * COLS * len(KS), dt, torch.get_num_threads()


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference's CPU path (its torch / numpy
    operations restated in oracle/, bit-exact with the reference on the
    golden vectors) on the host cores of rank 0; other ranks exit without
    work."""
    if rank != 0:
        return
    threads = use_all_host_threads()
    W, H = make_inputs(0)
    rows = args.cpu_rows
    for _ in range(args.warmup):
        cpu_reference_sample(W, H, rows)
    tot_w, tot_t = 0, 0.0
    for _ in range(args.steps):
        w, t, _ = cpu_reference_sample(W, H, rows)
        tot_w += w
        tot_t += t
    value = tot_w / tot_t
    sample = f"first {rows} rows of the 4096x4096 tensor ({rows * COLS} weights) at k=3 and k=2 per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_t / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         **host_info()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# measured peaks and per-kernel rooflines
# ---------------------------------------------------------------------------
def fp32_lane_peak(lib, dev, iters: int = 40000):
    """Measured FP32 lane rate (uq_fp32_lane_probe, packed f32x2 sub/mul/add
    chains on every SM): best of three launches after one warm-up."""
    import ctypes
    import torch
    from ultraquant_b200 import _device as D, _lib
    st = D.stream_handle(dev)
    ops = ctypes.c_double()
    out = {}
    for mode, name in ((0, "packed_f32x2"), (1, "scalar_f32")):
        _lib.check(lib.uq_fp32_lane_probe(mode, iters, ctypes.addressof(ops), st), "fp32 probe")
        best = 0.0
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            _lib.check(lib.uq_fp32_lane_probe(mode, iters, ctypes.addressof(ops), st), "fp32 probe")
            e1.record()
            torch.cuda.synchronize()
            best = max(best, ops.value / (e0.elapsed_time(e1) * 1e-3))
        out[name] = best / 1e12
    return out


def hbm_kernel_rooflines():
    """RHT / iRHT (fp64, 4096 columns and ffn_down's 14336 padded to 16384)
    and the E8 quantizer at config 3's rotated shape (4096 x 16384, step
    0.48): CUDA-event time per launch, L2 flushed between launches."""
    from ultraquant_b200 import profile_case as PC
    peak, src = measured_peaks()
    cases = [("rht", 4096, 4096, 0), ("irht", 4096, 4096, 0), ("rht", 4096, 16384, 14336),
             ("irht", 4096, 16384, 14336), ("e8", 4096, 16384, 0)]
    out = []
    for k, rows, n, n0 in cases:
        rec = PC.measure(k, rows=rows, n=n, n0=n0, iters=5, hbm_peak=peak)
        # rows of 16384 run both halves in one CTA (rht_halves_kernel)
        base = "rht_halves_kernel" if n == 16384 else "rht_tma_kernel"
        kern = {"rht": f"{base} (forward)", "irht": f"{base} (inverse)", "e8": "e8_tma_kernel"}[k]
        out.append({"kernel": kern, "shape": f"{rows}x{n0 or n}" + (f" (padded to {n})" if n0 else ""),
                    "dtype": "f64", "bound": "hbm", "achieved": rec["achieved_gbs"], "peak": peak, "unit": "GB/s",
                    "frac": rec["achieved_gbs"] / peak, "peak_source": src,
                    "bytes_per_launch": rec["algorithmic_bytes"], "ms_per_launch": rec["ms_per_run"]})
    return out


def scale_search_timing():
    """Config 3's opt-in per-row search over 16 E8 steps (uq_e8_scale_search)
    on the rotated ffn_down shape 4096 x 16384 fp64 at base step 0.48: CUDA
    events around the whole call (search kernel, host choice of lam, per-row
    decode) and per kernel."""
    import ctypes
    import torch
    from ultraquant_b200 import _device as D, _lib
    lib = _lib.load()
    dev = D.device()
    st = D.stream_handle(dev)
    rows, n = 4096, 16384
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(rows, n, dtype=torch.float64, device=dev, generator=g) * 0.015
    rec = torch.empty_like(A)
    ch = torch.empty(rows, dtype=torch.int32, device=dev)
    lam = ctypes.c_double()
    ws = D.workspace(lib.uq_e8_scale_search_workspace_bytes(rows, n), dev)

    def run():
        _lib.check(lib.uq_e8_scale_search(A.data_ptr(), rows, n, 0.48, rec.data_ptr(), None, ch.data_ptr(),
                                          ctypes.addressof(lam), ws.data_ptr(), ws.numel(), st), "scale search")
    run()
    torch.cuda.synchronize()
    lib.uq_profile_reset()
    lib.uq_profile_enable(1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        run()
    e1.record()
    torch.cuda.synchronize()
    lib.uq_profile_enable(0)
    per = {}
    for scope in ("e8_search", "e8_rowstep"):
        t, c = ctypes.c_double(), ctypes.c_int64()
        _lib.check(lib.uq_profile_read(scope.encode(), ctypes.byref(t), ctypes.byref(c)), "profile")
        per[scope] = t.value / 3
    lib.uq_profile_reset()
    ms = e0.elapsed_time(e1) / 3
    del A, rec
    return {"shape": f"{rows}x{n} fp64 (rotated ffn_down)", "candidates": 16, "base_step": 0.48,
            "ms_per_call": ms, "ms_search_kernel": per["e8_search"], "ms_rowstep_kernel": per["e8_rowstep"],
            "weights_per_s": rows * n / (ms * 1e-3),
            "candidate_decodes_per_s": 16 * rows * n / (per["e8_search"] * 1e-3)}


# ---------------------------------------------------------------------------
# default workload: the 4096 x 4096 tensor at k=3 and k=2, row-split
# ---------------------------------------------------------------------------
def workload_config(world: int):
    return {
        "workload": ("4096x4096 f32 N(0,0.02^2)+0.1% 8-sigma outliers (seed 0), lognormal(0,1) imatrix; "
                     "importance-weighted RHT(fp64) + bitshift-trellis Viterbi L=16 T=256 at k=3 and k=2, "
                     "scale group 256, decode, iRHT, packed codes; rows split across ranks, NCCL all-gather of "
                     "packed codes + scales + error sums"),
        "rows": ROWS, "cols": COLS, "L": L_BITS, "k": list(KS), "T": SEG, "scale_group": GROUP,
        "weights_per_step": ROWS * COLS * len(KS),
        "parallelism": f"row blocks of {ROWS // world} rows x{world} ranks" + (" + all-gather" if world > 1 else ""),
        "l2": "working set > L2: 8 KiB of backpointers per weight written each step",
    }


def run_tensor(args, rank: int, world: int, local: int):
    import ctypes
    import numpy as np
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from ultraquant_b200 import _lib, shard
    lib = _lib.load()

    specs = [shard.TensorSpec(f"w.k{R}", ROWS, COLS, L=L_BITS, R=R) for R in KS]
    block = -(-ROWS // world)
    plan = shard.plan(specs, world, block_rows=block)
    mine = [s for s in plan if s.rank == rank]
    W, H = make_inputs(0)
    r0 = min(s.row0 for s in mine) if mine else 0
    r1 = max(s.row1 for s in mine) if mine else 0
    Wd = torch.from_numpy(W[r0:r1]).to(dev)          # this rank's rows (device-resident)
    Hd = torch.from_numpy(H).to(dev)

    def weights_dev(s):
        return Wd[s.row0 - r0:s.row1 - r0], Hd

    def step():
        loc = shard.quantize_shards(plan, rank, weights_dev, SEG, GROUP)
        return shard.gather_codes(loc, plan, world, SEG, GROUP)

    def barrier():
        if world > 1:
            dist.barrier()

    clk = ClockSampler(phys_gpu_index(local)).__enter__()
    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    # ---- timed region (device events, max over ranks) ----------------------
    lib.uq_profile_reset()
    lib.uq_profile_enable(1)
    barrier()
    torch.cuda.synchronize()
    launches0 = int(lib.uq_launch_count())
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clk.mark(True)
    e0.record()
    out = None
    for _ in range(args.steps):
        out = step()
    e1.record()
    torch.cuda.synchronize()
    clk.mark(False)
    clk.__exit__(None, None, None)
    launches = int(lib.uq_launch_count()) - launches0
    lib.uq_profile_enable(0)
    ms = e0.elapsed_time(e1)
    vt, vn = ctypes.c_double(), ctypes.c_int64()
    _lib.check(lib.uq_profile_read(b"viterbi_fwd", ctypes.addressof(vt), ctypes.addressof(vn)), "profile")
    lib.uq_profile_reset()
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    weights = ROWS * COLS * len(KS) * args.steps
    value = weights / (ms_max / 1e3)

    # ---- Viterbi roofline against the measured FP32 lane peak --------------
    peak = fp32_lane_peak(lib, dev)
    props = torch.cuda.get_device_properties(dev)
    n_sm = props.multi_processor_count
    clocks = clk.summary()
    sm_max = (clocks or {}).get("sm_max_mhz") or 1965.0
    nominal = n_sm * 128 * sm_max * 1e6 / 1e12
    my_ops = sum(ops_per_weight(L_BITS, s.tensor.R) * s.rows * COLS for s in mine) * args.steps
    vit_s = vt.value / 1e3
    achieved = my_ops / vit_s / 1e12 if vit_s > 0 else 0.0
    my_seqs = sum(s.rows * COLS // SEG for s in mine) * args.steps
    roofline = {
        "kernel": "viterbi_fwd_kernel", "bound": "fp32_alu", "achieved": achieved, "peak": peak["packed_f32x2"],
        "unit": "Tops/s", "frac": achieved / peak["packed_f32x2"],
        "peak_source": "measured: uq_fp32_lane_probe (packed f32x2 sub/mul/add chains, all SMs, CUDA events, "
                       "same process, best of 3)",
        "peak_scalar_f32": peak["scalar_f32"], "nominal_peak": nominal, "frac_of_nominal": achieved / nominal,
        "ops_per_weight": {f"k{R}": ops_per_weight(L_BITS, R) for R in KS},
        "launches": int(vn.value), "kernel_ms_total": vt.value, "share_of_step": vt.value / ms if ms else None,
        # DRAM bytes per launch: one ncu capture of 296 sequences per k
        # (dram__bytes_read.sum + dram__bytes_write.sum), scaled by the
        # sequences of this run's launches (the traffic is the backpointers,
        # proportional to the sequences)
        "traffic": (sum(NCU_DRAM_BYTES_PER_SEQ[s.tensor.R] * s.rows * COLS // SEG for s in mine) * args.steps
                    / max(1, int(vn.value))),
        "traffic_unit": "bytes per launch",
        "traffic_source": "ncu capture, 296 sequences per k, scaled by the sequences per launch",
        # backpointer bytes: 2^L / 64 two-word records (8 B) per step and sequence
        "algorithmic_bytes_per_launch": my_seqs * (SEG - 1) * (1 << L_BITS) // 8 / max(1, int(vn.value)),
    }
    if clocks and clocks.get("sm_mhz"):
        roofline["sm_mhz_median"] = clocks["sm_mhz"]

    # ---- end to end through the public API with host buffers ---------------
    e2e = None
    if not args.no_e2e:
        Wp = torch.from_numpy(W[r0:r1]).pin_memory()
        Hp = torch.from_numpy(H)

        def weights_host(s):
            return Wp[s.row0 - r0:s.row1 - r0], Hp

        what_host = {(s.tensor.name, s.row0): torch.empty((s.rows, COLS), dtype=torch.float32, pin_memory=True)
                     for s in mine}
        ref = step()
        code_host = {k: (torch.empty(v.codes.shape, dtype=torch.int32, pin_memory=True),
                         torch.empty(v.sc.shape, dtype=torch.float32, pin_memory=True),
                         torch.empty(2, dtype=torch.float64, pin_memory=True)) for k, v in ref.items()}

        def e2e_step():
            loc = shard.quantize_shards(plan, rank, weights_host, SEG, GROUP, keep_what=True)
            res = shard.gather_codes(loc, plan, world, SEG, GROUP)
            for c in loc:
                what_host[(c.shard.tensor.name, c.shard.row0)].copy_(c.What, non_blocking=True)
            if rank == 0:
                for k, v in res.items():
                    hc, hs, he = code_host[k]
                    hc.copy_(v.codes, non_blocking=True)
                    hs.copy_(v.sc, non_blocking=True)
                    he.copy_(v.err, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        e2e_step()
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            e2e_step()
        t1.record()
        torch.cuda.synchronize()
        ems = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        h2d = sum(s.rows * COLS * 4 + H.nbytes for s in mine)
        d2h = sum(s.rows * COLS * 4 for s in mine)
        if rank == 0:
            d2h += sum(hc.numel() * 4 + hs.numel() * 4 + 16 for hc, hs, _ in code_host.values())
        e2e = {"value": weights / (float(ems.item()) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "ultraquant_b200.shard.quantize_shards(pinned host rows) + gather_codes -> "
                      "pinned host What rows and (rank 0) packed codes, scales, error sums"}
        # the e2e outputs equal the device-resident step's
        for k, v in ref.items():
            if rank == 0:
                assert torch.equal(code_host[k][0], v.codes.cpu()), "e2e codes differ from the device-resident run"

    cpu = None
    kern_roof = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = use_all_host_threads()
        w, t, _ = cpu_reference_sample(W, H, args.cpu_rows)
        cpu = {"value": w / t, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"first {args.cpu_rows} rows ({args.cpu_rows * COLS} weights) at k=3 and k=2, "
                         "oracle restatement of the reference torch CPU path", **host_info()}
    search = None
    if rank == 0 and not args.no_kernel_rooflines:
        kern_roof = hbm_kernel_rooflines()
        search = scale_search_timing()

    if world > 1:
        dist.barrier()
    if rank == 0:
        cfg = workload_config(world)
        cfg["wnmse"] = {k: v.wnmse for k, v in out.items()}
        cfg["packed_code_bytes"] = {k: v.codes.numel() * 4 for k, v in out.items()}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "roofline": roofline, "roofline_kernels": kern_roof, "e8_scale_search": search,
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# whole weight sets: Llama-3.1-8B (config 4) and Llama-3-70B (config 5)
# ---------------------------------------------------------------------------
def _student_t_block(g, rows, cols, std, dev):
    import torch
    z = torch.randn((rows, cols), generator=g, device=dev)
    chi = torch.randn((4, rows, cols), generator=g, device=dev).pow_(2).sum(0)
    return (z / torch.sqrt(chi / 4.0) / (2.0 ** 0.5) * std).float()


def run_weight_set(args, rank: int, world: int, local: int):
    """Whole Llama-shaped weight sets, sharded by tensor and row block
    (strong scaling: the set is fixed), trellis L=16 T=256; the run ends
    with every rank holding every tensor's packed codes, scales and error
    sums (one NCCL all-gather).

    llama8b : 32 x {q, o 4096 x 4096, k, v 1024 x 4096, gate, up 14336 x 4096,
              down 4096 x 14336}, Student-t(4) std 0.02, log-normal imatrix,
              k=3 on ffn_down / attn_q / attn_output, k=2 elsewhere.  Weights
              are generated on the device before the timed region.
    llama70b: 80 x {q, o 8192 x 8192, k, v 1024 x 8192, gate, up 28672 x 8192,
              down 8192 x 28672}, std 0.015, uniform k=2.  The set (274 GB in
              f32) does not fit the GPUs at 2 ranks, so each rank streams its
              row blocks: a block's weights are generated on the device just
              before the block is quantized (standing in for the read from
              host memory) and freed after it, inside the timed region."""
    import ctypes
    import torch
    import torch.distributed as dist
    from ultraquant_b200 import _lib, shard
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    lib = _lib.load()
    stream_blocks = args.workload == "llama70b"
    if args.workload == "llama70b":
        specs = shard.llama_shapes(layers=args.layers, hidden=8192, kv=1024, ffn=28672,
                                   k_by_type={t: 2 for t in ("attn_q", "attn_k", "attn_v", "attn_output",
                                                             "ffn_gate", "ffn_up", "ffn_down")})
        std = 0.015
        model = "Llama-3-70B"
    else:
        specs = shard.llama_shapes(layers=args.layers)
        std = 0.02
        model = "Llama-3.1-8B"
    plan = shard.plan(specs, world)
    mine = [s for s in plan if s.rank == rank]
    Hs = {}

    def H_of(spec):
        if spec.name not in Hs:
            gh = torch.Generator(device=dev)
            gh.manual_seed(sum(map(ord, spec.name)))
            Hs[spec.name] = torch.exp(torch.randn(spec.cols, generator=gh, device=dev, dtype=torch.float64))
        return Hs[spec.name]

    def gen(s):
        g = torch.Generator(device=dev)
        g.manual_seed(sum(map(ord, s.tensor.name)) * 1000 + s.row0)
        return _student_t_block(g, s.rows, s.tensor.cols, std, dev)

    data = {} if stream_blocks else {(s.tensor.name, s.row0): gen(s) for s in mine}
    for s in mine:
        H_of(s.tensor)
    # untimed warm-up: one block of every (padded width, k) this rank holds,
    # so the pipeline's workspace and the allocator's pools exist before timing
    warm = {}
    for s in mine:
        warm.setdefault((s.tensor.padded_cols, s.tensor.R), s)
    shard.quantize_shards(list(warm.values()), rank, lambda s: (gen(s), H_of(s.tensor)), SEG, GROUP)
    torch.cuda.synchronize()

    def weights(s):
        W = gen(s) if stream_blocks else data[(s.tensor.name, s.row0)]
        return W, Hs[s.tensor.name]

    clk = ClockSampler(phys_gpu_index(local)).__enter__()
    time.sleep(2.0)                       # nvidia-smi start-up outside the timed region
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    lib.uq_profile_reset()
    lib.uq_profile_enable(1)
    launches0 = int(lib.uq_launch_count())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.mark(True)
    e0.record()
    loc = shard.quantize_shards(plan, rank, weights, SEG, GROUP)
    out = shard.gather_codes(loc, plan, world, SEG, GROUP)
    e1.record()
    torch.cuda.synchronize()
    clk.mark(False)
    clk.__exit__(None, None, None)
    launches = int(lib.uq_launch_count()) - launches0
    lib.uq_profile_enable(0)
    vt, vn = ctypes.c_double(), ctypes.c_int64()
    _lib.check(lib.uq_profile_read(b"viterbi_fwd", ctypes.addressof(vt), ctypes.addressof(vn)), "profile")
    lib.uq_profile_reset()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    wall = float(ms.item()) / 1e3
    weights_n = sum(s.rows * s.cols for s in specs)
    peak = fp32_lane_peak(lib, dev)
    my_ops = sum(ops_per_weight(s.tensor.L, s.tensor.R) * s.rows * s.tensor.padded_cols for s in mine)
    achieved = my_ops / (vt.value / 1e3) / 1e12 if vt.value > 0 else 0.0
    roofline = {"kernel": "viterbi_fwd_kernel", "bound": "fp32_alu", "achieved": achieved,
                "peak": peak["packed_f32x2"], "unit": "Tops/s", "frac": achieved / peak["packed_f32x2"],
                "peak_source": "measured: uq_fp32_lane_probe (packed f32x2), rank 0",
                "launches": int(vn.value), "kernel_ms_total": vt.value,
                "share_of_step": vt.value / (wall * 1e3) if wall else None}
    # ---- end to end (llama8b): the rank's blocks from pinned host memory,
    # the gathered codes, scales and error sums read back on rank 0 ---------
    e2e = None
    if not stream_blocks and not args.no_e2e:
        host = {key: W.cpu().pin_memory() for key, W in data.items()}
        data.clear()
        torch.cuda.empty_cache()
        code_host = {k: (torch.empty(v.codes.shape, dtype=torch.int32, pin_memory=True),
                         torch.empty(v.sc.shape, dtype=torch.float32, pin_memory=True),
                         torch.empty(2, dtype=torch.float64, pin_memory=True)) for k, v in out.items()} \
            if rank == 0 else {}

        def weights_host(s):
            return host[(s.tensor.name, s.row0)], Hs[s.tensor.name]

        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        loc2 = shard.quantize_shards(plan, rank, weights_host, SEG, GROUP)
        out2 = shard.gather_codes(loc2, plan, world, SEG, GROUP)
        for k, (hc, hs, he) in code_host.items():
            hc.copy_(out2[k].codes, non_blocking=True)
            hs.copy_(out2[k].sc, non_blocking=True)
            he.copy_(out2[k].err, non_blocking=True)
        t1.record()
        torch.cuda.synchronize()
        ems = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        h2d = sum(s.rows * s.tensor.cols * 4 for s in mine)        # the imatrix stays on the device
        d2h = sum(hc.numel() * 4 + hs.numel() * 4 + 16 for hc, hs, _ in code_host.values())
        e2e = {"value": weights_n / (float(ems.item()) / 1e3), "unit": UNIT, "wall_s": float(ems.item()) / 1e3,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "ultraquant_b200.shard.quantize_shards(pinned host blocks) + gather_codes -> (rank 0) "
                      "pinned host packed codes, scales, error sums"}
        if rank == 0:
            for k in list(out)[:4]:
                assert torch.equal(code_host[k][0], out[k].codes.cpu()), "e2e codes differ from the resident run"
        del loc2, out2
    if world > 1:
        dist.barrier()
    if rank == 0:
        wn = {k: v.wnmse for k, v in out.items()}
        line = {"metric": f"{model}-shaped weight set trellis-quantized weights/sec (L=16, T=256)",
                "value": weights_n / wall, "unit": UNIT, "n_gpus": world, "steps": 1, "warmup": 0,
                "ms_per_step": wall * 1e3, "wall_s": wall, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"{model}-shaped weight set, {args.layers} layers, {len(specs)} tensors"
                                       + (", row blocks streamed (generated per block on the device)"
                                          if stream_blocks else ", weights resident before timing"),
                           "weights": weights_n, "layers": args.layers, "L": 16, "T": SEG,
                           "parallelism": f"tensor x row-block plan over {world} ranks + all-gather of packed codes",
                           "target": "< 60 s on 8 B200 for the Llama-3.1-8B set" if model == "Llama-3.1-8B" else None},
                "wnmse_mean": {t: sum(v for n, v in wn.items() if f".{t}." in n) /
                               max(1, sum(1 for n in wn if f".{t}." in n))
                               for t in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up",
                                         "ffn_down")},
                "packed_code_bytes": sum(v.codes.numel() * 4 for v in out.values()),
                "roofline": roofline, "e2e": e2e,
                "e2e_note": None if e2e else "row blocks generated on the device per block (no host copy of the "
                                             "274 GB set)",
                "gpu_launches": launches, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=8, help="rows of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-kernel-rooflines", action="store_true", help="skip the RHT / E8 roofline entries")
    ap.add_argument("--workload", default="tensor", choices=["tensor", "llama8b", "llama70b"],
                    help="tensor: the 4096x4096 L=16 k=3+2 step (default); llama8b / llama70b: the "
                         "whole Llama-3.1-8B- / Llama-3-70B-shaped weight set sharded over the ranks (one step)")
    ap.add_argument("--layers", type=int, default=None,
                    help="layers of the llama workloads (default 32 for llama8b, 80 for llama70b)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload in ("llama8b", "llama70b"):
        if args.layers is None:
            args.layers = 80 if args.workload == "llama70b" else 32
        return run_weight_set(args, rank, world, local)
    return run_tensor(args, rank, world, local)


if __name__ == "__main__":
    main()
