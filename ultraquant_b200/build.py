"""Build ``libuq_b200.so`` (the C-ABI library) for sm_100a with nvcc.

Run ``python -m ultraquant_b200.build`` (or ``__graft_entry__.build()``).
Objects go to ``ultraquant_b200/_build/``; the shared library is written next
to this file so that it travels with the source tree.

Flags: ``-fmad=false`` keeps every multiply and add separately rounded
(bit-exact with the element-wise numpy / torch reference); divisions and
square roots stay IEEE (no fast-math).  The CUDA runtime is linked statically,
so the library only needs the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libuq_b200.so")

SOURCES = ["uq_host.cpp", "uq_rht.cu", "uq_e8.cu", "uq_trellis.cu", "uq_pipeline.cu", "uq_qat.cu", "uq_q8.cu", "uq_qe8.cu", "uq_peak.cu", "uq_e8search.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-O2", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(OUT, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "uq_b200.h"))
    objs, jobs = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(OUT, src + ".o")
        objs.append(obj)
        if not _stale(obj, [path] + headers) and not ptxas_info:
            continue
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", path, "-o", obj]
        if ptxas_info and src.endswith(".cu"):
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        jobs.append((src, cmd))

    def compile_one(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    # one nvcc per translation unit, in parallel
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for err in ex.map(compile_one, jobs):
            if ptxas_info:
                sys.stderr.write(err)
    if _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="-v" in sys.argv))
