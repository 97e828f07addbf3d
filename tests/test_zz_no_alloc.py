"""The scratch-free Viterbi entry point (uq_trellis_viterbi_noalloc).

It serves callers that cannot allocate device memory themselves -- a host
program whose own allocator owns the GPU and gives plug-ins no allocation
hook, or a latency-critical path that must not hit cudaMalloc's implicit
synchronisation.  Its backpointer scratch is a fixed static device array, so
the test checks that it returns exactly the states of the workspace entry
point and of the oracle's Viterbi (the C restatement of trellis.py:84-105),
on two calls in a row (the second call finds the array holding the first
call's contents), through the C ABI.  At L = 16 and T = 256 the array holds
64 sequences, so the 130- and 150-sequence cases run several full batches and
a partial last one.  This file is collected last on purpose; it also passes
when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _states_workspace(lib, D, xn, L, R):
    import torch
    nseq, T = xn.shape
    cw = D.codebook(L, xn.device)
    out = torch.empty((nseq, T), dtype=torch.int32, device=xn.device)
    ws = torch.empty(lib.uq_trellis_workspace_bytes(nseq, T, L, R), dtype=torch.uint8, device=xn.device)
    rc = lib.uq_trellis_viterbi(xn.data_ptr(), nseq, T, L, R, cw.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                ws.numel(), D.stream_handle(xn.device))
    assert rc == 0, lib.uq_last_error()
    return out


def _states_noalloc(lib, D, xn, L, R):
    import torch
    nseq, T = xn.shape
    cw = D.codebook(L, xn.device)
    out = torch.full((nseq, T), -1, dtype=torch.int32, device=xn.device)
    rc = lib.uq_trellis_viterbi_noalloc(xn.data_ptr(), nseq, T, L, R, cw.data_ptr(), out.data_ptr(),
                                        D.stream_handle(xn.device))
    assert rc == 0, lib.uq_last_error()
    return out


@pytest.mark.parametrize("L,R,nseq", [(12, 2, 3000), (16, 2, 150), (16, 2, 130), (16, 3, 70)])
def test_noalloc_matches_workspace_entry_point(L, R, nseq):
    import torch
    from oracle import cviterbi
    from ultraquant_b200 import _device as D
    from ultraquant_b200 import _lib
    lib = _lib.load()
    assert lib.uq_trellis_noalloc_scratch_bytes() == 64 << 20
    torch.manual_seed(L * 10 + R + nseq)
    for call in range(2):
        x = torch.randn(nseq, 256, device="cuda")
        x[: 2 + call] = torch.round(x[: 2 + call] * 2) / 2     # exact values: cost ties
        ref = _states_workspace(lib, D, x, L, R)
        got = _states_noalloc(lib, D, x, L, R)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: states differ from the workspace entry point"
        oracle = cviterbi.viterbi_segments_c(x.cpu().numpy(), L, R)
        assert np.array_equal(got.cpu().numpy(), oracle), f"call {call}: states differ from the oracle"
    assert lib.uq_device_errors(D.stream_handle(D.device())) == 0


def test_noalloc_rejects_oversized_sequence():
    from ultraquant_b200 import _lib
    lib = _lib.load()
    # T = 20000 at L = 16 needs ~80 MB of backpointers for one sequence
    rc = lib.uq_trellis_viterbi_noalloc(ctypes.c_void_p(16), 1, 20000, 16, 2, ctypes.c_void_p(16),
                                        ctypes.c_void_p(16), None)
    assert rc == _lib.UQ_ERR_INVALID
    assert b"static array" in lib.uq_last_error()
