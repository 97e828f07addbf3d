"""Single-kernel cases for profiling and per-kernel rooflines.

    python -m ultraquant_b200.profile_case <kernel> [--rows R] [--n N] [--L L] [--R K] [--iters I]

Each case builds seeded inputs on the GPU, runs the kernel once untimed and
then ``--iters`` times, and prints one JSON line with the kernel's device
time (CUDA events recorded around each launch on its stream) and its
achieved rate against the algorithmic bytes (HBM-bound kernels) or lane
operations (the Viterbi forward).  With ``--iters 0`` it only runs the
kernel once, which is the form to put under ``ncu -k <kernel> -c 1``.

Kernels: viterbi (segments of 256, L / R), rht and irht (fp64), e8,
normalize, fwht (fp32), recon and recon_bwd (the QAT decoder, fp32), q8enc and
q8dec (Q8_0 blocks, fp32 side), rht28 (opt-in unpadded 28 x P transform, --n0),
qe8 (finite-codebook E8, fp64, --bpw; all of its kernels), e8search (the opt-in
per-row search over 16 E8 steps at base step 0.48, fp64; the search kernel).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _device as D
from . import _lib

# profiler scope name of each case's kernel
SCOPE = {"viterbi": "viterbi_fwd", "rht": "rht", "irht": "rht", "e8": "e8_quant",
         "normalize": "normalize", "fwht": "fwht", "recon": "qat_recon", "recon_bwd": "qat_recon_bwd",
         "q8enc": "q8_encode", "q8dec": "q8_decode", "rht28": "rht", "qe8": "qe8_search",
         "e8search": "e8_search"}


def _peaks():
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk.get("hbm_gbs") or pk.get("hbm_GBs") or 6650.0), "measured"
    except (OSError, ValueError, TypeError):
        return 6650.0, "fallback"


def build_case(args, lib, st):
    """Returns (run() -> None, units of work per run, unit name)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    dev = D.device()
    rows, n = args.rows, args.n
    n0 = args.n0 or n
    npad = 1 << (n0 - 1).bit_length()
    signs = D.signs(npad, 0, dev)
    k = args.kernel
    if k == "viterbi":
        L, R, nseq = args.L, args.R, args.rows
        x = torch.randn(nseq, 256, device=dev, generator=g)
        cw = D.codebook(L, dev)
        states = torch.empty((nseq, 256), dtype=torch.int32, device=dev)
        ws = D.workspace(lib.uq_trellis_workspace_bytes(nseq, 256, L, R), dev)

        def run():
            _lib.check(lib.uq_trellis_viterbi(x.data_ptr(), nseq, 256, L, R, cw.data_ptr(), states.data_ptr(),
                                              ws.data_ptr(), ws.numel(), st), "viterbi")
        ops = 3 * (1 << L) + ((1 << R) - 1) * (1 << (L - R))
        return run, nseq * 256 * ops, "lane_ops"
    if k in ("rht", "irht"):
        if k == "irht":
            X = torch.randn(rows, npad, dtype=torch.float64, device=dev, generator=g)
            out = torch.empty(rows, n0, dtype=torch.float64, device=dev)

            def run():
                _lib.check(lib.uq_irht_rows(X.data_ptr(), 1, rows, npad, npad, n0, signs.data_ptr(),
                                            out.data_ptr(), st), "irht")
            return run, rows * npad * 8 + rows * n0 * 8, "bytes"
        A = torch.randn(rows, n0, dtype=torch.float64, device=dev, generator=g)
        out = torch.empty(rows, npad, dtype=torch.float64, device=dev)

        def run():
            _lib.check(lib.uq_rht_rows(A.data_ptr(), 1, rows, n0, n0, signs.data_ptr(), out.data_ptr(), st), "rht")
        return run, rows * n0 * 8 + rows * npad * 8, "bytes"
    if k == "e8":
        X = torch.randn(rows, n, dtype=torch.float64, device=dev, generator=g)
        rec = torch.empty_like(X)

        def run():
            _lib.check(lib.uq_e8_quant(X.data_ptr(), 1, X.numel(), 256, 0.48, rec.data_ptr(), None, st), "e8")
        return run, X.numel() * 16, "bytes"
    if k == "normalize":
        x = torch.randn(rows * n, device=dev, generator=g)
        xn = torch.empty_like(x)
        sc = torch.empty(x.numel() // 256, device=dev)

        def run():
            _lib.check(lib.uq_trellis_normalize(x.data_ptr(), 0, x.numel(), 256, 256, xn.data_ptr(), sc.data_ptr(),
                                                st), "normalize")
        return run, x.numel() * 8 + sc.numel() * 4, "bytes"
    if k == "fwht":
        x = torch.randn(rows, n, device=dev, generator=g)
        out = torch.empty_like(x)

        def run():
            _lib.check(lib.uq_fwht(x.data_ptr(), 0, rows, n, n, n, None, None, 0, out.data_ptr(), n, n, st), "fwht")
        return run, x.numel() * 8, "bytes"
    if k in ("recon", "recon_bwd"):
        L = args.L
        cw = D.codebook(L, dev)
        states = torch.randint(0, 1 << L, (rows * n,), dtype=torch.int32, device=dev, generator=g)
        sc = torch.rand(rows * n // 256, device=dev, generator=g) + 0.1
        sH = torch.rand(n, device=dev, generator=g) + 0.5
        s32 = signs.float()
        if k == "recon":
            out = torch.empty(rows, n, device=dev)

            def run():
                _lib.check(lib.uq_qat_recon(states.data_ptr(), 0, rows, n, cw.data_ptr(), cw.numel(), sc.data_ptr(),
                                            256, s32.data_ptr(), sH.data_ptr(), n, out.data_ptr(), n, st), "recon")
            return run, rows * n * 8, "bytes"
        gr = torch.randn(rows, n, device=dev, generator=g)
        gcw, gsc = torch.empty_like(cw), torch.empty_like(sc)
        ws = D.workspace(lib.uq_qat_recon_backward_workspace_bytes(cw.numel(), sc.numel()), dev)

        def run():
            _lib.check(lib.uq_qat_recon_backward(gr.data_ptr(), n, states.data_ptr(), 0, rows, n, cw.data_ptr(),
                                                 cw.numel(), sc.data_ptr(), sc.numel(), 256, s32.data_ptr(),
                                                 sH.data_ptr(), n, gcw.data_ptr(), gsc.data_ptr(), ws.data_ptr(),
                                                 ws.numel(), st), "recon_bwd")
        return run, rows * n * 8, "bytes"
    if k == "rht28":
        A = torch.randn(rows, n0, dtype=torch.float64, device=dev, generator=g)
        out = torch.empty_like(A)
        d28 = D.signs(n0, 0, dev)

        def run():
            _lib.check(lib.uq_rht28_rows(A.data_ptr(), 1, rows, n0, n0, None, d28.data_ptr(), out.data_ptr(), st), "rht28")
        return run, rows * n0 * 16, "bytes"
    if k == "e8search":
        import ctypes
        A = torch.randn(rows, n, dtype=torch.float64, device=dev, generator=g) * 0.015
        rec = torch.empty_like(A)
        ch = torch.empty(rows, dtype=torch.int32, device=dev)
        lam = ctypes.c_double()
        ws = D.workspace(lib.uq_e8_scale_search_workspace_bytes(rows, n), dev)

        def run():
            _lib.check(lib.uq_e8_scale_search(A.data_ptr(), rows, n, 0.48, rec.data_ptr(), None, ch.data_ptr(),
                                              ctypes.addressof(lam), ws.data_ptr(), ws.numel(), st), "e8search")
        # the search kernel reads the row once per candidate (16 x 8 B per weight)
        return run, A.numel() * 8 * 16, "bytes"
    if k == "qe8":
        from . import qlab as Q
        A = torch.randn(rows, n, dtype=torch.float64, device=dev, generator=g) * 0.02
        K = 1 << int(round(args.bpw * 8))
        cb, cb32, scale, cut = Q._e8_codebook_dev(K, dev)
        out = torch.empty_like(A)
        ws = D.workspace(lib.uq_q_e8_workspace_bytes(A.numel(), 256), dev)

        def run():
            _lib.check(lib.uq_q_e8(A.data_ptr(), 1, A.numel(), 256, cb.data_ptr(), cb32.data_ptr(), cb.shape[0],
                                   scale, cut, out.data_ptr(), ws.data_ptr(), ws.numel(), st), "qe8")
        return run, A.numel() * 16, "bytes"
    if k in ("q8enc", "q8dec"):
        W = torch.randn(rows, n, device=dev, generator=g) * 0.02
        q = torch.empty((rows, n // 32 * 34), dtype=torch.uint8, device=dev)
        _lib.check(lib.uq_q8_encode(W.data_ptr(), 0, rows, n, n, q.data_ptr(), st), "q8enc")
        if k == "q8enc":
            def run():
                _lib.check(lib.uq_q8_encode(W.data_ptr(), 0, rows, n, n, q.data_ptr(), st), "q8enc")
        else:
            def run():
                _lib.check(lib.uq_q8_decode(q.data_ptr(), rows, n, W.data_ptr(), n, st), "q8dec")
        return run, rows * n * 4 + rows * n // 32 * 34, "bytes"
    raise SystemExit(f"unknown kernel {k}")


def measure(kernel: str, rows: int = 4096, n: int = 4096, n0: int = 0, L: int = 16, R: int = 2, bpw: float = 2.0,
            iters: int = 10, hbm_peak: float | None = None) -> dict:
    """Time one case: a warm-up launch, then ``iters`` runs with a buffer
    larger than L2 rewritten before each (cold inputs), CUDA events around
    every launch of the case's kernel.  Returns the JSON record of main()."""
    args = argparse.Namespace(kernel=kernel, rows=rows, n=n, n0=n0, L=L, R=R, bpw=bpw, iters=iters)
    lib = _lib.load()
    dev = D.device()
    st = D.stream_handle(dev)
    run, units, unit = build_case(args, lib, st)
    run()
    torch.cuda.synchronize()
    if iters <= 0:
        return {"kernel": kernel, "ok": True}
    # a buffer larger than L2 rewritten between launches keeps the inputs cold
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    lib.uq_profile_enable(1)
    lib.uq_profile_reset()
    for _ in range(iters):
        flush.fill_(1)
        run()
    torch.cuda.synchronize()
    tot = _lib.ctypes.c_double(0.0)
    cnt = _lib.ctypes.c_int64(0)
    _lib.check(lib.uq_profile_read(SCOPE[kernel].encode(), _lib.ctypes.byref(tot), _lib.ctypes.byref(cnt)),
               "profile")
    rec = {"kernel": kernel, "rows": rows, "n": n0 or n, "runs": iters, "launches": cnt.value}
    if kernel == "qe8":
        # every kernel of the call, and the call as a whole (events on the stream)
        for scope in ("e8_quant", "qe8_cb_norm", "qe8_classify", "qe8_search", "qe8_exact"):
            t, c = _lib.ctypes.c_double(0.0), _lib.ctypes.c_int64(0)
            _lib.check(lib.uq_profile_read(scope.encode(), _lib.ctypes.byref(t), _lib.ctypes.byref(c)), "profile")
            rec[f"ms_{scope}"] = t.value / iters
        lib.uq_profile_enable(0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush.fill_(1)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        rec["ms_call"] = e0.elapsed_time(e1)
        rec["bpw"] = bpw
        rec["weights_per_s"] = rows * n / (rec["ms_call"] * 1e-3)
    lib.uq_profile_enable(0)
    lib.uq_profile_reset()
    _lib.check(lib.uq_device_errors(st), kernel)
    ms = tot.value / iters            # device time of the kernel per run (all its launches)
    rec["ms_per_run"] = ms
    if unit == "bytes":
        peak, kind = (hbm_peak, "given") if hbm_peak else _peaks()
        gbs = units / (ms * 1e-3) / 1e9
        rec.update(algorithmic_bytes=units, achieved_gbs=gbs, peak_gbs=peak, frac=gbs / peak, peak_kind=kind)
    else:
        props = torch.cuda.get_device_properties(dev)
        nominal = props.multi_processor_count * 128 * 1965e6
        tops = units / (ms * 1e-3)
        rec.update(lane_ops=units, achieved_tops=tops / 1e12, frac_of_nominal_fp32=tops / nominal, L=L, R=R)
    return rec


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("kernel", choices=sorted(SCOPE))
    ap.add_argument("--rows", type=int, default=4096, help="rows (sequences for viterbi)")
    ap.add_argument("--n", type=int, default=4096, help="row width (power of two)")
    ap.add_argument("--n0", type=int, default=0, help="unpadded width of rht / irht (default n)")
    ap.add_argument("--L", type=int, default=16)
    ap.add_argument("--R", type=int, default=2)
    ap.add_argument("--bpw", type=float, default=2.0, help="rate of the qe8 case")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    print(json.dumps(measure(args.kernel, args.rows, args.n, args.n0, args.L, args.R, args.bpw, args.iters)))


if __name__ == "__main__":
    main()
