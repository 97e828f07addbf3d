"""NVTX ranges of the pipeline stages and kernel launches.

The library pushes a range in the "ultraquant_b200" domain around every
pipeline entry point (uq_quant_trellis, uq_quant_e8, ...), every stage
(rht_forward, trellis_normalize, trellis_viterbi, trellis_decode,
rht_inverse, e8_quant, e8_scale_search) and every kernel launch.  The tests
load a small NVTX injection library (nvtx_recorder.c, beside this file)
through NVTX_INJECTION64_PATH in a child process and read back the ranges it
saw.  NVTX initialises once per process at its first call, so each case
runs in a fresh interpreter.
"""
import os
import subprocess
import sys
import textwrap

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
SRC = os.path.join(HERE, "nvtx_recorder.c")
CUDA_INC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")


@pytest.fixture(scope="module")
def recorder(tmp_path_factory):
    out = tmp_path_factory.mktemp("nvtx") / "libnvtx_recorder.so"
    r = subprocess.run(["gcc", "-O1", "-fPIC", "-shared", f"-I{CUDA_INC}", SRC, "-o", str(out)],
                       capture_output=True, text=True)
    if r.returncode:
        pytest.fail(f"gcc failed for nvtx_recorder.c:\n{r.stderr}")
    return str(out)


def _record(recorder, tmp_path, code):
    log = tmp_path / "nvtx.log"
    env = dict(os.environ, NVTX_INJECTION64_PATH=recorder, UQ_NVTX_RECORD=str(log))
    r = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    return log.read_text().splitlines() if log.exists() else []


def _ranges(lines):
    """(depth, name, parent) of every pushed range, in push order; checks
    that every push has its pop."""
    out, stack = [], []
    for ln in lines:
        if ln.startswith("+"):
            out.append((len(stack), ln[1:], stack[-1] if stack else None))
            stack.append(ln[1:])
        elif ln == "-":
            assert stack, "pop without a push"
            stack.pop()
    assert not stack, f"ranges left open: {stack}"
    return out


def _is_subsequence(want, seq):
    it = iter(seq)
    return all(any(w == s for s in it) for w in want)


def test_entry_point_ranges_without_a_device(recorder, tmp_path):
    """An empty matrix and a rejected shape return before any CUDA call, but
    their ranges still open and close: the library is linked with NVTX and a
    tool attached through NVTX_INJECTION64_PATH sees its domain."""
    lines = _record(recorder, tmp_path, """
        from ultraquant_b200 import _lib
        lib = _lib.load()
        # rows = 0: valid, nothing to do
        assert lib.uq_quant_trellis(None, 0, 0, 256, 256, None, 12, 2, 256, 256, None, None, None, None,
                                    None, None, None, 0, None) == 0
        # rows = -1: rejected
        assert lib.uq_quant_e8(None, 0, -1, 256, 256, None, 0.5, 256, None, None, None, None, None, 0,
                               None) != 0
    """)
    assert "domain ultraquant_b200" in lines
    r = _ranges(lines)
    assert [(d, n) for d, n, _ in r] == [(0, "uq_quant_trellis"), (0, "uq_quant_e8")]


def test_no_tool_no_record(tmp_path):
    """Without NVTX_INJECTION64_PATH nothing is loaded and nothing recorded."""
    log = tmp_path / "nvtx.log"
    env = {k: v for k, v in os.environ.items() if k != "NVTX_INJECTION64_PATH"}
    env["UQ_NVTX_RECORD"] = str(log)
    r = subprocess.run([sys.executable, "-c", "from ultraquant_b200 import _lib; lib = _lib.load(); "
                        "lib.uq_quant_trellis(None, 0, 0, 256, 256, None, 12, 2, 256, 256, None, None, None, "
                        "None, None, None, None, 0, None)"], cwd=REPO, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    assert not log.exists()


@pytest.mark.gpu
def test_trellis_pipeline_stage_ranges(recorder, tmp_path):
    """uq_quant_trellis on a 64 x 256 matrix: its stages in order, each
    holding the ranges of its own kernel launches."""
    lines = _record(recorder, tmp_path, """
        import torch
        from ultraquant_b200 import pipeline
        g = torch.Generator(device="cuda").manual_seed(0)
        W = torch.randn(64, 256, device="cuda", generator=g) * 0.02
        H = torch.ones(256, dtype=torch.float64, device="cuda")
        pipeline.quant_trellis_device(W, H, L=8, R=2, seg=64)
        torch.cuda.synchronize()
    """)
    r = _ranges(lines)
    top = [i for i, (d, n, _) in enumerate(r) if n == "uq_quant_trellis"]
    assert len(top) == 1
    stages = [n for d, n, p in r if p == "uq_quant_trellis"]
    assert _is_subsequence(["importance_scale", "rht_forward", "trellis_normalize", "trellis_viterbi",
                            "trellis_decode", "rht_inverse"], stages), stages
    kids = lambda stage: {n for _, n, p in r if p == stage}
    assert "rht" in kids("rht_forward")
    assert "normalize" in kids("trellis_normalize")
    assert {"viterbi_fwd", "traceback"} <= kids("trellis_viterbi")
    assert "decode" in kids("trellis_decode")
    assert "rht" in kids("rht_inverse")


@pytest.mark.gpu
def test_e8_pipeline_stage_ranges(recorder, tmp_path):
    """uq_quant_e8 and the opt-in scale search on a 32 x 512 matrix."""
    lines = _record(recorder, tmp_path, """
        import torch
        from ultraquant_b200 import pipeline
        g = torch.Generator(device="cuda").manual_seed(1)
        W = torch.randn(32, 512, device="cuda", generator=g) * 0.02
        H = torch.ones(512, dtype=torch.float64, device="cuda")
        pipeline.quant_step_device(W, H, 0.5)
        pipeline.quant_step_device(W, H, 0.5, scale_search=True)
        torch.cuda.synchronize()
    """)
    r = _ranges(lines)
    assert _is_subsequence(["rht_forward", "e8_quant", "rht_inverse"],
                           [n for _, n, p in r if p == "uq_quant_e8"])
    assert _is_subsequence(["rht_forward", "e8_scale_search", "rht_inverse"],
                           [n for _, n, p in r if p == "uq_quant_e8_search"])
    assert any(p == "e8_quant" for _, _, p in r)
    assert any(p == "e8_scale_search" for _, _, p in r)
