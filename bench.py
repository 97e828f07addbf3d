#!/usr/bin/env python
"""Benchmark: trellis-quantized weights/s on B200.

Workload (the configuration the metric is quoted on, single GPU): a
4096 x 4096 float32 weight matrix, N(0, 0.02^2) from seed 0 with 0.1 % of the
entries replaced by +-8 sigma outliers, and a log-normal(0, 1) per-column
imatrix.  One step runs the importance-weighted trellis recipe of
buildtrellis.py -- A = W*sqrt(H), RHT (fp64), per-256 RMS, Viterbi with
L = 16 state bits and T = 256, decode, inverse RHT, /sqrt(H), weighted-error
statistics -- once at k = 2 and once at k = 3 bits/weight.  Synthetic, seeded
inputs stand in for real checkpoints.

value     : weights quantized per second (both k), inputs resident in HBM.
e2e       : the same through the public host API (pinned host W in, host
            What out, copies inside the timed region).
roofline  : the Viterbi forward kernel against the FP32 lane peak, timed
            live with CUDA events around its launches.
cpu_baseline / --impl reference : the CPU restatement of the reference's
            torch path (oracle/) on the host cores, on a bounded row sample.

Multi-GPU (torchrun): every rank quantizes its own tensor (seed = rank, as the
tensors of a model are independent); per-tensor error statistics are
all-gathered over NCCL.  Time = max over ranks; value = all ranks' weights /
that time ("weak" scaling).
"""
from __future__ import annotations

import argparse
import json
import os
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
KS = (2, 3)
SEG = 256
GROUP = 256
# ncu capture of viterbi_fwd_kernel<2,2> (profiles/viterbi_l16r2_ncu.md): DRAM
# bytes per processed weight, used to scale to one full launch.
NCU_TRAFFIC_BYTES_PER_WEIGHT = None


def make_inputs(seed: int):
    import numpy as np
    rng = np.random.RandomState(seed)
    W = rng.normal(0.0, 0.02, size=(ROWS, COLS))
    m = rng.random_sample(W.shape) < 0.001
    W[m] = np.sign(rng.normal(size=int(m.sum()))) * 8 * 0.02
    H = np.exp(rng.normal(0.0, 1.0, size=COLS))
    return W.astype(np.float32), H


# ncu (L=16, T=256, one launch of 296 sequences): DRAM read + write bytes
NCU_DRAM_BYTES_PER_SEQ = {2: (1.252352e6 + 251.667968e6) / 296, 3: (1.233152e6 + 251.116544e6) / 296}


def ops_per_weight(L: int, R: int) -> int:
    """Algorithmic lane ops of one Viterbi step per weight: sub, mul, add per
    state plus (2^R - 1) compares per predecessor group."""
    return 3 * (1 << L) + ((1 << R) - 1) * (1 << (L - R))


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

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
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_reference_sample(W, H, rows: int):
    """Oracle restatement of the reference path on `rows` rows (k=2 and k=3)."""
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
    """--impl reference: the reference's CPU path (restated in oracle/) on the
    host cores of rank 0; other ranks exit without work."""
    if rank != 0:
        return
    W, H = make_inputs(0)
    rows = args.cpu_rows
    for _ in range(args.warmup):
        cpu_reference_sample(W, H, rows)
    tot_w, tot_t, cores = 0, 0.0, 1
    for _ in range(args.steps):
        w, t, cores = cpu_reference_sample(W, H, rows)
        tot_w += w
        tot_t += t
    value = tot_w / tot_t
    sample = f"first {rows} rows of the 4096x4096 tensor ({rows * COLS} weights) at k=2 and k=3 per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_llama8b(args, rank: int, world: int, local: int):
    """Whole Llama-3.1-8B-shaped weight set (32 x {q, k, v, o 4096/1024 x 4096,
    gate/up 14336 x 4096, down 4096 x 14336}), Student-t(4) weights with std
    0.02 and log-normal imatrix, trellis L=16 T=256 with k=3 on ffn_down /
    attn_q / attn_output and k=2 elsewhere, sharded by tensor and row block
    (strong scaling: the set is fixed).  ``--workload llama70b``: the
    Llama-3-70B shapes (hidden 8192, k/v 1024 x 8192, ffn 28672), std 0.015,
    uniform k=2.  Weights are generated on the device before the timed region."""
    import torch
    import torch.distributed as dist
    from ultraquant_b200 import pipeline, shard
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    if args.workload == "llama70b":
        specs = shard.llama_shapes(layers=args.layers, hidden=8192, kv=1024, ffn=28672,
                                   k_by_type={t: 2 for t in ("attn_q", "attn_k", "attn_v", "attn_output",
                                                             "ffn_gate", "ffn_up", "ffn_down")})
        std = 0.015
    else:
        specs = shard.llama_shapes(layers=args.layers)
        std = 0.02
    plan = [s for s in shard.plan(specs, world) if s.rank == rank]
    data = []
    for sh in plan:
        g = torch.Generator(device=dev)
        g.manual_seed(sum(map(ord, sh.tensor.name)) * 1000 + sh.row0)
        z = torch.randn((sh.rows, sh.tensor.cols), generator=g, device=dev)
        chi = torch.randn((4, sh.rows, sh.tensor.cols), generator=g, device=dev).pow_(2).sum(0)
        W = (z / torch.sqrt(chi / 4.0) / (2.0 ** 0.5) * std).float()
        gh = torch.Generator(device=dev)
        gh.manual_seed(sum(map(ord, sh.tensor.name)))
        H = torch.exp(torch.randn(sh.tensor.cols, generator=gh, device=dev, dtype=torch.float64))
        data.append((sh, W, H))
        del z, chi
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    results = []
    for sh, W, H in data:
        r = pipeline.quant_trellis_device(W, H, L=16, R=sh.tensor.R, seg=SEG, scale_group=GROUP, keep_codes=False)
        results.append(shard.ShardResult(sh, r.What, r.err))
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    wn = shard.gather_errors(results, specs)
    weights = sum(s.rows * s.cols for s in specs)
    if rank == 0:
        model = "Llama-3-70B" if args.workload == "llama70b" else "Llama-3.1-8B"
        line = {"metric": f"{model}-shaped weight set trellis-quantized, wall time on device",
                "value": float(ms.item()) / 1e3, "unit": "s", "n_gpus": world, "steps": 1, "warmup": 0,
                "higher_is_better": False, "scaling": "strong", "weights": weights,
                "weights_per_s": weights / (float(ms.item()) / 1e3), "layers": args.layers,
                "wnmse_mean": {k: sum(v for n, v in wn.items() if f".{k}." in n) / max(1, sum(1 for n in wn if f".{k}." in n))
                               for k in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")},
                "dtype": "f32", "data": "synthetic"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def workload_config(world: int):
    return {
        "workload": ("4096x4096 f32 N(0,0.02^2)+0.1% 8-sigma outliers (seed=rank), lognormal(0,1) imatrix; "
                     "importance-weighted RHT(fp64) + bitshift-trellis Viterbi L=16 T=256 at k=2 and k=3, "
                     "scale group 256, decode, iRHT"),
        "rows": ROWS, "cols": COLS, "L": L_BITS, "k": list(KS), "T": SEG, "scale_group": GROUP,
        "weights_per_step_per_gpu": ROWS * COLS * len(KS),
        "parallelism": f"one tensor per rank x{world}",
        "l2": "working set > L2: 4 KiB of backpointers per weight written each step",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=8, help="rows of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--workload", default="tensor", choices=["tensor", "llama8b", "llama70b"],
                    help="tensor: the 4096x4096 L=16 k=2+3 step (default); llama8b / llama70b: the "
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
        return run_llama8b(args, rank, world, local)

    import numpy as np
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from ultraquant_b200 import _lib, pipeline
    lib = _lib.load()

    W, H = make_inputs(rank)
    Wd = torch.from_numpy(W).to(dev)
    Hd = torch.from_numpy(H).to(dev)

    def step():
        errs = []
        for R in KS:
            r = pipeline.quant_trellis_device(Wd, Hd, L=L_BITS, R=R, seg=SEG, scale_group=GROUP)
            errs.append(r.err)
        return errs

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    # ---- timed region (device events, max over ranks) ----------------------
    lib.uq_profile_reset()
    lib.uq_profile_enable(1)
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys_idx = int(phys.split(",")[local]) if phys and phys.split(",")[local].strip().isdigit() else local
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(phys_idx) as clk:
        e0.record()
        errs = None
        for _ in range(args.steps):
            errs = step()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    lib.uq_profile_enable(0)
    launches = int(lib.uq_launch_count())
    ms = e0.elapsed_time(e1)
    import ctypes
    vt, vn = ctypes.c_double(), ctypes.c_int64()
    _lib.check(lib.uq_profile_read(b"viterbi_fwd", ctypes.addressof(vt), ctypes.addressof(vn)), "profile")
    lib.uq_profile_reset()
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        # the path's only exchange: per-tensor error statistics of every rank
        gathered = [torch.zeros(2 * len(KS), dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(gathered, torch.cat(errs))
    ms_max = float(ms_t.item())
    weights = ROWS * COLS * len(KS) * args.steps * world
    value = weights / (ms_max / 1e3)

    # ---- roofline of the Viterbi forward kernel ---------------------------
    props = torch.cuda.get_device_properties(dev)
    n_sm = props.multi_processor_count
    clocks = clk.summary()
    sm_max = (clocks or {}).get("sm_max_mhz") or 1965.0
    peak_tops = n_sm * 128 * sm_max * 1e6 / 1e12
    vit_ops = sum(ops_per_weight(L_BITS, R) for R in KS) * ROWS * COLS * args.steps
    vit_s = vt.value / 1e3
    achieved = vit_ops / vit_s / 1e12 if vit_s > 0 else 0.0
    roofline = {
        "kernel": "viterbi_fwd_kernel", "bound": "fp32_alu", "achieved": achieved, "peak": peak_tops,
        "unit": "Tops/s", "frac": achieved / peak_tops,
        "peak_source": f"nominal FP32 lanes: {n_sm} SMs x 128 x {sm_max:.0f} MHz (no measured FP32 peak on file)",
        "ops_per_weight": {f"k{R}": ops_per_weight(L_BITS, R) for R in KS},
        "launches": int(vn.value), "kernel_ms_total": vt.value, "share_of_step": vt.value / ms if ms else None,
        # DRAM bytes per launch: one ncu capture of 296 sequences per k
        # (dram__bytes_read.sum + dram__bytes_write.sum), scaled by the
        # sequences of the bench's launches (the traffic is the backpointers,
        # proportional to the sequences)
        "traffic": (sum(NCU_DRAM_BYTES_PER_SEQ[R] for R in KS) / len(KS)
                    * (ROWS * COLS // SEG) * len(KS) * args.steps / max(1, int(vn.value))),
        "traffic_unit": "bytes per launch",
        "traffic_source": "ncu capture, 296 sequences per k, scaled by sequences per launch",
    }
    if clocks and clocks.get("sm_mhz"):
        roofline["frac_at_measured_clock"] = achieved / (n_sm * 128 * clocks["sm_mhz"] * 1e6 / 1e12)

    # ---- end to end through the public host API ---------------------------
    e2e = None
    if not args.no_e2e:
        Wp = torch.from_numpy(W).pin_memory()
        Hp = torch.from_numpy(H)
        pipeline.quant_trellis(Wp, Hp, L=L_BITS, R=KS[0], seg=SEG, scale_group=GROUP)
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            for R in KS:
                pipeline.quant_trellis(Wp, Hp, L=L_BITS, R=R, seg=SEG, scale_group=GROUP)
        t1.record()
        torch.cuda.synchronize()
        ems = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": weights / (float(ems.item()) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": len(KS) * (W.nbytes + H.nbytes),
               "d2h_bytes_per_step": len(KS) * W.nbytes,
               "api": "ultraquant_b200.pipeline.quant_trellis(pinned host W, host H) -> pinned host What"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        w, t, cores = cpu_reference_sample(W, H, args.cpu_rows)
        cpu = {"value": w / t, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"first {args.cpu_rows} rows ({args.cpu_rows * COLS} weights) at k=2 and k=3, "
                         "oracle restatement of the reference torch CPU path"}

    if world > 1:
        dist.barrier()
    if rank == 0:
        err = torch.cat(errs).double().cpu().numpy()
        cfg = workload_config(world)
        cfg["wnmse"] = {f"k{R}": float(err[2 * i] / err[2 * i + 1]) for i, R in enumerate(KS)}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
